#!/usr/bin/env python
"""Decode throughput of libcortex on B200: generated tokens per second.

Headline workload (the d=1024 configuration of the metric): a seeded
d=1024, 2-layer, 16-head, ctx-1024, V=16384 SNAI_V4 model (fp32 weights
N(0, 0.02), unit RMSNorm weights), 4096 independent sequences split evenly
over the ranks, prompts of 512 uniform random ids, then 512 decode steps at
positions 512..1023 with the reference's top-k/top-p sampler (variant of
src/tensor_ffi_adapter.php:168-204: T=0.7, top_k=40, top_p=0.9, subtractive
repetition penalty 1.1 over every token fed so far) and seeded per-step
uniform draws; projections run on tcgen05 tensor cores with bf16 operands and
fp32 accumulation; the KV cache is fp32.

A step is one decode step of every local sequence (sample one id from the
current logits, feed it).  The cost of a step grows with the position (the
attention reads every cached position), so the --steps timed steps sit
around the job's mean position: after the prompt, untimed decode steps
bring the sequences to 768 - (steps - 1) / 2 - warmup, then --warmup steps,
then the timed steps (mean position 767.5, the mean of 512..1023).  With
--steps 512 or more the timed steps cover the whole generation (rewinding
to 512 at the context limit).  The KV cache (68.7 GB on one GPU) is far
larger than L2, so no L2 flush is needed.

`value`: the timed steps through the device-pointer API, one captured
decode step replayed as a CUDA graph per step (cortex_decode_steps), timed
with CUDA events on the engine's stream.  `e2e`: the same steps through the
host-pointer C-ABI call (uniforms in, ids out each step).  Per-kernel times
(`kernels`, `roofline`) come from a separate profiled pass over the same
positions (CUDA events around every launch).  `ids_sha256`: a digest of the
timed steps' ids of all 4096 sequences in sequence order, gathered to rank
0's host without NCCL (pinned device-to-host copies, then a gloo gather);
it is the same for every number of GPUs.

Multi-GPU: one process per GPU under torchrun, no collective on the data
path; the max over ranks of the device time is reported.  Scaling is
strong: the 4096 sequences are split over the ranks.

With one GPU the line also carries, as extra keys, the other workloads of
the metric: `c3` (d=512, 512 sequences), `c2` (d=256 Net2Net-upscaled
model, 64 sequences), `sampling` (the isolated sampler workload, GB/s
against the HBM peak) and `gemv_pass` (the one-row fp32 decode pass the PHP
host drives, GB/s with L2 flushed before each pass).

--impl reference times the oracle port of the reference's CPU engine
(oracle/snai_oracle.c: core/cortex.nim forward + the PHP sampler, libm exp)
on all host threads over a bounded sample at the same positions.
"""
import argparse
import hashlib
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

V = 16384
CTX = 1024
NOMINAL_HBM_GBS = 7700.0  # B200 HGX datasheet figure, for context beside the measured copy peak

# The configurations of the metric.  c4 is the headline; c3 and c2 run as
# extra keys of the one-GPU line (or alone with --config).
CONFIGS = {
    "c4": dict(D=1024, L=2, HEADS=16, PROMPT=512, GEN=512, SEQS=4096, VARIANT=1, T=0.7, REP=1.1, TOP_K=40,
               TOP_P=0.9, model="seeded SNAI_V4 d1024 L2 heads16 (init_base layout, N(0,0.02))",
               workload="d=1024 L=2 heads=16 V=16384 ctx=1024, 4096 sequences, prompt 512 + 512 decode steps, "
                        "top-k 40 / top-p 0.9 / T 0.7 / rep 1.1 sampling"),
    "c3": dict(D=512, L=2, HEADS=8, PROMPT=512, GEN=512, SEQS=512, VARIANT=1, T=0.7, REP=1.1, TOP_K=40,
               TOP_P=0.9, model="seeded SNAI_V4 d512 L2 heads8 (init_base layout, N(0,0.02))",
               workload="d=512 L=2 heads=8 V=16384 ctx=1024, 512 sequences, prompt 512 + 512 decode steps, "
                        "top-k 40 / top-p 0.9 / T 0.7 / rep 1.1 sampling"),
    "c2": dict(D=256, L=4, HEADS=4, PROMPT=256, GEN=256, SEQS=64, VARIANT=0, T=0.8, REP=1.15, TOP_K=40,
               TOP_P=0.9, model="SNAI_V4 d256 L4 ctx1024: seeded Net2Net upscale of the seeded d128 L2 ctx512 drone",
               workload="d=256 L=4 heads=4 V=16384 ctx=1024 (upscaled drone), 64 sequences, prompt 256 + 256 "
                        "decode steps, variant-A sampling T 0.8 / rep 1.15"),
}
PARALLELISM = "independent sequences sharded over the ranks (no collective on the data path)"


def metric_name(c):
    return f"generated tokens/sec (d={c['D']} decode)"


def config_dict(c):
    return {"workload": c["workload"], "model": c["model"], "global_batch": c["SEQS"], "seq_len": CTX,
            "prompt": c["PROMPT"], "gemm": "tcgen05 bf16 x bf16 -> fp32",
            "kv_cache": "fp32",
            "l2": "inputs larger than L2 (KV cache %.1f GB in all)" % (c["SEQS"] * c["L"] * 2 * CTX * c["D"] * 4 / 1e9),
            "parallelism": PARALLELISM}


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm": float(p["hbm_gbs"]), "bf16": float(p["bf16_tflops"]),
                "bf16_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), "kind": "measured"}
    except Exception:
        return {"hbm": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "kind": "fallback"}


def bench_dir():
    return os.environ.get("SNAI_BENCH_DIR", tempfile.gettempdir())


def make_model(name, rank=0):
    """The configuration's model file (seeded; written once per host)."""
    from snai_b200 import modelgen
    c = CONFIGS[name]
    D, L = c["D"], c["L"]
    if name == "c2":
        drone = os.path.join(bench_dir(), f"snai_bench_drone_d128_L2_seed1234_r{rank}.snai")
        if not os.path.exists(drone) or os.path.getsize(drone) != modelgen.expected_size(V, 128, 512, 2):
            modelgen.random_model(drone, V, 128, 512, 2, seed=1234, std=0.02)
        p = os.path.join(bench_dir(), f"snai_bench_c2_up256_r{rank}.snai")
        if not os.path.exists(p) or os.path.getsize(p) != modelgen.expected_size(V, D, 4 * D, L):
            from snai_b200 import upscale_file
            upscale_file(drone, p, D, seed=4321)  # Net2Net upscale on the GPU
        return p
    p = os.path.join(bench_dir(), f"snai_bench_d{D}_L{L}_seed1234_r{rank}.snai")
    if not os.path.exists(p) or os.path.getsize(p) != modelgen.expected_size(V, D, 4 * D, L):
        modelgen.random_model(p, V, D, CTX, L, seed=1234, std=0.02)
    return p


def window(c, steps, warmup):
    """(first untimed position, first timed position): the timed steps centred
    on the job's mean decode position, within prompt..ctx when they fit."""
    lo, hi = c["PROMPT"], c["PROMPT"] + c["GEN"]  # decode steps feed positions lo..hi-1
    mean = (lo + hi - 1) / 2.0
    p0 = int(round(mean - (steps - 1) / 2.0))
    if p0 - warmup < lo or p0 + steps > hi:
        return lo, lo + warmup  # the whole generation (rewinds past the end)
    return p0 - warmup, p0


class ClockSampler:
    """SM clocks and clock-event reasons sampled every 10 ms through NVML
    (nvidia-smi at its fastest loop as a fallback)."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown"}

    def __init__(self, gpus, period=0.01):
        self.gpus = gpus
        self.period = period
        self.samples = []  # (sm_mhz, max_mhz, reasons bitmask)
        self.stop = threading.Event()
        self.proc = None
        self.nvml = None

    def __enter__(self):
        if not self.gpus:
            return self
        try:
            import pynvml
            pynvml.nvmlInit()
            hs = []
            for g in self.gpus:
                hs.append(pynvml.nvmlDeviceGetHandleByUUID(g) if g.startswith("GPU-")
                          else pynvml.nvmlDeviceGetHandleByIndex(int(g)))
            self.nvml = (pynvml, hs)
            self.t = threading.Thread(target=self._poll_nvml, daemon=True)
            self.t.start()
            return self
        except Exception:
            self.nvml = None
        try:
            fields = "clocks.sm,clocks.max.sm,clocks_event_reasons.active"
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={fields}", "--format=csv,noheader,nounits",
                                          "-lms", "20", "-i", ",".join(self.gpus)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read_smi, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _poll_nvml(self):
        nv, hs = self.nvml
        while not self.stop.is_set():
            for h in hs:
                try:
                    sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                    mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
                    try:
                        rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                    except Exception:
                        rs = nv.nvmlDeviceGetCurrentClocksThrottleReasons(h)
                    self.samples.append((float(sm), float(mx), int(rs)))
                except Exception:
                    pass
            time.sleep(self.period)

    def _read_smi(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            try:
                self.samples.append((float(parts[0]), float(parts[1]), int(parts[2], 16)))
            except (ValueError, IndexError):
                continue

    def __exit__(self, *a):
        self.stop.set()
        if self.nvml:
            self.t.join(timeout=1)
            try:
                self.nvml[0].nvmlShutdown()
            except Exception:
                pass
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [s[0] for s in self.samples]
        reasons = sorted({n for s in self.samples for bit, n in self.REASONS.items() if s[2] & bit})
        return {"sm_mhz": float(np.median(sm)), "sm_min_mhz": min(sm), "sm_max_mhz": max(s[1] for s in self.samples),
                "reasons": reasons, "samples": len(sm),
                "source": "nvml every 10 ms" if self.nvml else "nvidia-smi -lms 20",
                "span": "warm-up and timed steps"}


def visible_gpu_ids(n):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [x.strip() for x in vis.split(",") if x.strip()]
        return ids[:n]
    return [str(i) for i in range(n)]


def cpu_sample(name, steps_timed, nthreads, start_pos, nseq=None, warmup=1):
    """Times the oracle port (one thread per sequence) for a bounded sample
    of decode steps from start_pos."""
    import oracle as O
    c = CONFIGS[name]
    o = O.Oracle(make_model(name), num_heads=c["HEADS"])
    nseq = nseq or nthreads
    b = o.batch(nseq, start_pos, seed=99)
    for _ in range(warmup):
        b.step(c["VARIANT"], c["T"], c["REP"], c["TOP_K"], c["TOP_P"], nthreads)
    secs = 0.0
    for _ in range(steps_timed):
        secs += b.step(c["VARIANT"], c["T"], c["REP"], c["TOP_K"], c["TOP_P"], nthreads)
    b.close()
    o.close()
    return nseq * steps_timed / secs, secs, nseq


def reference_arm(args, rank, world):
    """The reference's CPU path (oracle port) on all host threads."""
    if rank != 0:
        return
    c = CONFIGS[args.config]
    nthreads = os.cpu_count() or 1
    start, p0 = window(c, args.steps, args.warmup)
    rate, secs, nseq = cpu_sample(args.config, args.steps, nthreads, start, warmup=args.warmup)
    sample = (f"{nseq} sequences x {args.steps} decode steps at positions {p0}..{p0 + args.steps - 1} "
              f"(after {args.warmup} warm-up steps from {start}), one thread per sequence")
    line = {"impl": "reference", "metric": metric_name(c), "value": rate, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * secs / max(1, args.steps),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded model, random prompt ids)", "config": config_dict(c),
            "cpu_baseline": {"value": rate, "unit": "tokens/s", "cores": nthreads, "kind": "port", "sample": sample},
            "e2e": {"value": rate, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


class Dist:
    """Barriers, max-over-ranks (NCCL) and a host gather (gloo)."""

    def __init__(self, world, dev):
        self.world = world
        self.dev = dev
        self.gloo = None
        if world > 1:
            import torch.distributed as dist
            self.gloo = dist.new_group(backend="gloo")

    def barrier(self):
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier()

    def max(self, x):
        if self.world == 1:
            return x
        import torch
        import torch.distributed as dist
        t = torch.tensor([x], dtype=torch.float64, device=self.dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def gather_host(self, arr):
        """Rank 0 receives every rank's host array (same shape), in rank order."""
        if self.world == 1:
            return [arr]
        import torch
        import torch.distributed as dist
        t = torch.from_numpy(np.ascontiguousarray(arr))
        out = [torch.empty_like(t) for _ in range(self.world)] if dist.get_rank() == 0 else None
        dist.gather(t, out, dst=0, group=self.gloo)
        return None if out is None else [o.numpy() for o in out]


def decode_run(name, args, rank, world, local_rank, dist_, peaks, extra=False):
    """One decode configuration: prefill, centred warm-up and timed steps
    (graph replay), a profiled pass and the host-pointer e2e pass.  Returns
    the measurements (rank 0) or None."""
    import torch
    from snai_b200 import PREC_BF16, Cortex, sample_params

    c = CONFIGS[name]
    total, D, PROMPT = c["SEQS"], c["D"], c["PROMPT"]
    dev = torch.device("cuda", local_rank)
    if total % world:
        raise SystemExit(f"{total} sequences do not split over {world} ranks")
    B = total // world
    path = make_model(name, rank)
    t_load = time.perf_counter()
    eng = Cortex(path, num_heads=c["HEADS"], max_seqs=B, device=local_rank, precision=PREC_BF16)
    load_s = time.perf_counter() - t_load
    stream = torch.cuda.Stream(device=dev)
    eng.set_stream(stream.cuda_stream)
    rng = np.random.default_rng(1234)
    prompts = rng.integers(0, V, (total, PROMPT)).astype(np.int32)[rank * B:(rank + 1) * B]
    start, p0 = window(c, args.steps, args.warmup)
    END = PROMPT + c["GEN"]  # the job decodes positions PROMPT..END-1
    ff = start - PROMPT  # untimed steps before the warm-up
    total_steps = ff + args.warmup + args.steps
    # per-step uniforms of every sequence, sliced per rank: the same draws for any number of GPUs
    U_all = rng.random((total_steps, total), dtype=np.float32)
    U = torch.from_numpy(np.ascontiguousarray(U_all[:, rank * B:(rank + 1) * B])).to(dev)
    prm = sample_params(c["VARIANT"], c["T"], c["REP"], c["TOP_K"], c["TOP_P"])

    # ---- prefill (reported separately) ----
    dist_.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    with torch.cuda.stream(stream):
        for s0 in range(0, B, 256):
            n = min(256, B - s0)
            toks = torch.from_numpy(np.ascontiguousarray(prompts[s0:s0 + n].ravel())).to(dev)
            eng.forward_dev(toks, n, PROMPT, slots=np.arange(s0, s0 + n))
    eng.synchronize()
    prefill_s = dist_.max(time.perf_counter() - t0)

    ids_buf = torch.zeros((max(total_steps, 1), B), dtype=torch.int32, device=dev)

    def steps_dev(i0, n):
        # n decode steps in one call (cortex_decode_steps: one captured step
        # replayed as a CUDA graph), rewinding to the prompt at the job's end
        while n > 0:
            if eng.pos(0) >= END:
                eng.rewind(PROMPT)
            k = min(n, END - eng.pos(0))
            eng.decode_steps_dev(U[i0:i0 + k], prm, ids_buf[i0:i0 + k])
            i0 += k
            n -= k

    # ---- untimed steps to the window, warm-up, timed steps (value) ----
    clk = ClockSampler(visible_gpu_ids(world) if rank == 0 else [])
    with torch.cuda.stream(stream):
        if ff:
            steps_dev(0, ff)
    eng.synchronize()
    with clk:
        with torch.cuda.stream(stream):
            steps_dev(ff, args.warmup)
        eng.synchronize()
        dist_.barrier()
        torch.cuda.synchronize()
        launches0 = eng.launches
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            torch.cuda.nvtx.range_push("timed")
            ev0.record(stream)
            steps_dev(ff + args.warmup, args.steps)
            ev1.record(stream)
            torch.cuda.nvtx.range_pop()
        ev1.synchronize()
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    launches = eng.launches - launches0
    dist_.barrier()
    ms_max = dist_.max(ms)

    # ids of the timed steps, to rank 0's host (pinned copy; gloo gather)
    host_ids = torch.empty((args.steps, B), dtype=torch.int32, pin_memory=True)
    host_ids.copy_(ids_buf[ff + args.warmup:ff + args.warmup + args.steps])
    parts = dist_.gather_host(host_ids.numpy())
    digest = None
    if rank == 0:
        digest = hashlib.sha256(np.ascontiguousarray(np.concatenate(parts, axis=1)).tobytes()).hexdigest()[:16]

    # ---- profiled pass over the same positions (per-launch CUDA events) ----
    n_prof = min(args.steps, 32)
    pp = p0 + (args.steps - n_prof) // 2
    if pp > END - n_prof or pp < PROMPT:
        pp = PROMPT
    eng.rewind(pp)
    eng.profile(True)
    with torch.cuda.stream(stream):
        for i in range(n_prof):
            eng.decode_dev(U[ff + args.warmup + i], prm, ids_buf[0])
    eng.synchronize()
    prof = eng.profile_read()
    eng.profile(False)

    # ---- end to end through the host-pointer C ABI (e2e), same positions ----
    eng.rewind(start)
    Uh = U_all[:, rank * B:(rank + 1) * B]
    out_ids = np.zeros(B, dtype=np.int32)

    def step_host(i):
        # one call per step from host memory (uniforms in, ids out), through
        # the graph-replayed decode
        if eng.pos(0) >= END:
            eng.rewind(PROMPT)
        out_ids[:] = eng.decode_steps(Uh[i:i + 1], prm)[0]

    for i in range(args.warmup):
        step_host(ff + i)
    dist_.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        step_host(ff + args.warmup + i)
    e1.record(stream)
    e1.synchronize()
    e2e_ms = dist_.max(e0.elapsed_time(e1))
    eng.close()
    del U, ids_buf
    torch.cuda.empty_cache()
    if rank != 0:
        return None

    tokens = total * args.steps
    att_n, att_ms, att_bytes, _ = prof["attention"]
    achieved = (att_bytes / att_n) / (att_ms / att_n / 1e3) / 1e9 if att_n else None
    # DRAM traffic per launch: the ratio of ncu-measured to algorithmic bytes
    # of a smaller capture (same kernel, traffic proportional to the KV
    # positions read) times this pass's algorithmic bytes per launch
    traffic = None
    tp = os.path.join(ROOT, "profiles", "attention_decode_traffic.json")
    if os.path.exists(tp) and att_n:
        try:
            traffic = json.load(open(tp))["traffic_per_algorithmic_byte"] * att_bytes / att_n
        except Exception:
            traffic = None
    total_prof_ms = sum(v[1] for v in prof.values()) or 1.0
    kernels = {}
    for k, v in prof.items():
        if not v[0]:
            continue
        kernels[k] = {"launches": v[0], "ms": round(v[1], 3), "share": round(v[1] / total_prof_ms, 4),
                      "GB/s": round(v[2] / (v[1] / 1e3) / 1e9, 1) if v[1] else None,
                      "TFLOP/s": round(v[3] / (v[1] / 1e3) / 1e12, 2) if v[1] and v[3] else None}
        if k in ("qkv", "wo", "up", "down", "logits") and v[1] and v[3]:
            kernels[k]["frac_bf16_sustained"] = round(v[3] / (v[1] / 1e3) / 1e12 / peaks["bf16_sustained"], 3)
        if k in ("attention", "sampler") and v[1]:
            kernels[k]["frac_hbm"] = round(v[2] / (v[1] / 1e3) / 1e9 / peaks["hbm"], 3)
    res = {
        "metric": metric_name(c), "value": tokens / (ms_max / 1e3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
        "positions": {"timed": [p0, p0 + args.steps - 1] if p0 + args.steps <= END
                      else f"{PROMPT}..{END - 1} (rewinds)",
                      "untimed_steps_before_warmup": ff},
        "e2e": {"value": tokens / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": 8 * B,
                "d2h_bytes_per_step": 4 * B, "api": "cortex_decode_steps(steps=1, SNAI_HOST_PTRS) per step"},
        "gpu_launches": int(launches),
        "roofline": {"kernel": "attention (decode, fp32 KV)", "bound": "hbm", "achieved": achieved,
                     "peak": peaks["hbm"], "unit": "GB/s", "frac": (achieved / peaks["hbm"]) if achieved else None,
                     "traffic": traffic, "peak_source": f"{peaks['kind']} hbm_gbs (a copy; a lower bound on HBM)",
                     "frac_of_nominal_7700": (achieved / NOMINAL_HBM_GBS) if achieved else None,
                     "algorithmic_bytes_per_launch": att_bytes / att_n if att_n else None,
                     "timing": f"per-launch CUDA events, profiled pass of {n_prof} steps from position {pp}"},
        "kernels": kernels,
        "ids_sha256": digest,
        "prefill": {"tokens_per_s": total * PROMPT / prefill_s, "seconds": prefill_s},
        "load_s": load_s,
        "clocks": clk.summary(),
    }
    return res


def sampling_lines(peaks, steps=10, warmup=3, check_rows=64, cpu_rows=256):
    """The isolated sampler workload: fp32 logits [8192, V], V in {16384,
    32000, 131072}, N(0, 4) (variance 4) with 1% of entries raised by 12, a
    256-id history per row, one uniform per row; greedy, variant A (T 0.7,
    rep 1.15) and variant B (T 0.7, top-k 50, top-p 0.95, rep 1.15).
    Algorithmic bytes per row: 4V (logits) + 4*256 (history) + 4 (uniform)
    + 4 (id); L2 flushed between timed launches.  Each line checks
    check_rows rows against the oracle (bit-exact ids)."""
    import torch

    import oracle as O
    from snai_b200 import VARIANT_A, VARIANT_B, sample_device, sample_params
    rows, H = 8192, 256
    dev = torch.device("cuda")
    modes = [("greedy", sample_params(VARIANT_A, 0.01, 1.15, nan_guard=0), (VARIANT_A, 0.01, 1.15, 40, 0.9)),
             ("A_T0.7", sample_params(VARIANT_A, 0.7, 1.15, nan_guard=0), (VARIANT_A, 0.7, 1.15, 40, 0.9)),
             ("B_T0.7_k50_p0.95", sample_params(VARIANT_B, 0.7, 1.15, 50, 0.95), (VARIANT_B, 0.7, 1.15, 50, 0.95))]
    out_lines = []
    for Vs in (16384, 32000, 131072):
        g = torch.Generator(device=dev).manual_seed(Vs)
        L = torch.randn(rows, Vs, device=dev, generator=g) * 2.0
        L += (torch.rand(rows, Vs, device=dev, generator=g) < 0.01).float() * 12.0
        hist = torch.randint(0, Vs, (rows, H), device=dev, generator=g, dtype=torch.int32)
        Ud = torch.rand(rows, device=dev, generator=g)
        out = torch.zeros(rows, dtype=torch.int32, device=dev)
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        for name, prm, oargs in modes:
            for _ in range(warmup):
                sample_device(L, Ud, prm, hist, None, out)
            ts = []
            for _ in range(steps):
                flush.zero_()  # 256 MB > L2 between timed launches
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                sample_device(L, Ud, prm, hist, None, out)
                e1.record()
                e1.synchronize()
                ts.append(e0.elapsed_time(e1))
            ms = float(np.median(ts))
            nbytes = rows * (4 * Vs + 4 * H + 8)
            gbs = nbytes / (ms / 1e3) / 1e9
            want, _ = O.sample_rows(L[:check_rows].cpu().numpy(), hist[:check_rows].cpu().numpy(),
                                    Ud[:check_rows].cpu().numpy(), *oargs, exp_mode=1)
            exact = bool(np.array_equal(out[:check_rows].cpu().numpy(), want))
            line = {"mode": name, "vocab": Vs, "rows": rows, "value": gbs, "unit": "GB/s", "ms": ms,
                    "rows_per_s": rows / (ms / 1e3),
                    "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm"], "unit": "GB/s",
                                 "frac": gbs / peaks["hbm"], "peak_source": f"{peaks['kind']} hbm_gbs"},
                    "l2": "flushed (256 MB written) before each timed launch",
                    f"bit_exact_vs_oracle_{check_rows}_rows": exact}
            if cpu_rows:
                _, rate = O.sample_rows(L[:cpu_rows].cpu().numpy(), hist[:cpu_rows].cpu().numpy(),
                                        Ud[:cpu_rows].cpu().numpy(), *oargs, exp_mode=0,
                                        nthreads=os.cpu_count() or 1)
                line["cpu_baseline"] = {"value": rate, "unit": "rows/s", "cores": os.cpu_count(), "kind": "port",
                                        "sample": f"{cpu_rows} rows"}
            out_lines.append(line)
        del L, hist, Ud, out, flush
        torch.cuda.empty_cache()
    return out_lines


def gemv_pass_line(peaks, passes=50, rows=1, pos=16, split=True, fused=False):
    """The small-batch path the PHP host drives: one decode pass of `rows`
    rows (embedding, 2 layers of fp32 GEMV projections and attention, final
    norm, logits) on the d=1024 benchmark model in FP32 mode, at position
    `pos` (each pass rewinds to it).  L2 is flushed (256 MB written) before
    each pass, so the fp32 weights (168 MB) stream from HBM; each pass is
    timed with its own CUDA events.  Bytes per pass are the library's
    algorithmic sums (weights once, KV read, activations).  split=False
    turns the split-position attention off (SNAI_ATTENTION_SPLIT=0) to
    compare; fused=True runs the pass as the persistent pass kernel
    (SNAI_PASS_KERNEL=1) instead of one kernel per stage."""
    import torch
    from snai_b200 import PREC_FP32, Cortex
    dev = torch.device("cuda")
    saved = {k: os.environ.get(k) for k in ("SNAI_ATTENTION_SPLIT", "SNAI_PASS_KERNEL")}
    # fused: the persistent pass kernel (opt-in in the library)
    os.environ["SNAI_ATTENTION_SPLIT"] = "1" if split else "0"
    os.environ["SNAI_PASS_KERNEL"] = "1" if fused else "0"
    try:
        eng = Cortex(make_model("c4"), num_heads=16, max_seqs=rows, precision=PREC_FP32)
    finally:
        for k, v in saved.items():
            if v is None:
                del os.environ[k]
            else:
                os.environ[k] = v
    stream = torch.cuda.Stream(device=dev)
    eng.set_stream(stream.cuda_stream)
    rng = np.random.default_rng(7)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    with torch.cuda.stream(stream):
        eng.forward_dev(torch.from_numpy(rng.integers(0, V, pos * rows).astype(np.int32)).to(dev), rows, pos)
        # algorithmic bytes and the attention time of one pass from the profiler
        eng.profile(True)
        for _ in range(3):
            eng.rewind(pos)
            flush.zero_()
            eng.forward_dev(torch.from_numpy(rng.integers(0, V, rows).astype(np.int32)).to(dev), rows, 1)
        eng.synchronize()
        prof = eng.profile_read()
        eng.profile(False)
        pass_bytes = sum(v[2] for v in prof.values()) / 3
        toks = [torch.from_numpy(rng.integers(0, V, rows).astype(np.int32)).to(dev) for _ in range(passes)]
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(passes)]
        for i, (a, b) in enumerate(ev):
            eng.rewind(pos)
            flush.zero_()
            # hold the stream so the pass is queued whole and its kernels run back to back
            torch.cuda._sleep(400000)
            a.record(stream)
            eng.forward_dev(toks[i], rows, 1)
            b.record(stream)
        eng.synchronize()
    us = sorted(1e3 * a.elapsed_time(b) for a, b in ev)[passes // 2]
    eng.close()
    del flush
    torch.cuda.empty_cache()
    gbs = pass_bytes / (us / 1e6) / 1e9
    att_n, att_ms, att_bytes, _ = prof["attention"]
    return {"metric": "one-row decode pass GB/s (fp32 GEMV path, d=1024)", "value": gbs, "unit": "GB/s",
            "rows": rows, "position": pos, "us_per_pass": us, "bytes_per_pass": pass_bytes, "passes": passes,
            "attention_us_per_launch": 1e3 * att_ms / att_n if att_n else None,
            "attention_split": split, "persistent_pass_kernel": bool(fused and prof["pass"][0]),
            "launches_per_pass": sum(v[0] for v in prof.values()) / 3,
            "timing": "median of per-pass CUDA events",
            "l2": "flushed (256 MB written) before each pass",
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm"], "unit": "GB/s",
                         "frac": gbs / peaks["hbm"], "peak_source": f"{peaks['kind']} hbm_gbs"}}


def train_flops(D, L, V, att_ch, M):
    """Algorithmic FLOPs of one training step over M positions: the
    projections forward (2 M (12 D^2 L + V D)) and twice that backward (the
    input and the weight gradient), causal attention 2 M^2 att_ch per layer
    forward (scores, weighted values) and 5 M^2 att_ch backward (scores
    again, dP, dQ, dK, dV)."""
    proj = 2.0 * M * (12.0 * D * D * L + V * D)
    return 3.0 * proj + 7.0 * M * M * att_ch * L


def train_line(peaks, name, steps=5, warmup=2, cpu_tokens=16, tf32=False):
    """cortex_train_step on the configuration's model: one sequence of ctx
    (1024) tokens per step, as the PHP training worker feeds it
    (src/train_worker.php:113-145), fp32.  `value` is tokens/s by CUDA events
    on the engine's stream around each call (host token arrays in, the loss
    out: the call's own copies are inside); `e2e` is the same by the host
    clock.  The CPU baseline is the oracle's step (one thread, like the
    reference) on the first cpu_tokens tokens.  tf32: a TF32 engine, whose
    projection GEMMs run on the tensor cores (the attention products stay
    fp32 SIMT)."""
    import torch
    import oracle as O
    from snai_b200 import PREC_FP32, PREC_TF32, Cortex
    c = CONFIGS[name]
    D, L, H = c["D"], c["L"], c["HEADS"]
    path = make_model(name)
    dev = torch.device("cuda")
    eng = Cortex(path, num_heads=H, max_seqs=1, precision=PREC_TF32 if tf32 else PREC_FP32)
    stream = torch.cuda.Stream(device=dev)
    eng.set_stream(stream.cuda_stream)
    rng = np.random.default_rng(11)
    M = CTX
    seqs = [rng.integers(0, V, M + 1).astype(np.int32) for _ in range(steps + warmup)]
    lr = 1e-4
    losses = []
    for i in range(warmup):
        eng.train_step(seqs[i][:-1], seqs[i][1:], lr)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    t0 = time.perf_counter()
    for i, (a, b) in enumerate(ev):
        x = seqs[warmup + i]
        a.record(stream)
        losses.append(eng.train_step(x[:-1], x[1:], lr))
        b.record(stream)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    ms = sum(a.elapsed_time(b) for a, b in ev) / steps
    launches = eng.launches
    eng.close()
    flops = train_flops(D, L, V, H * (D // H), M)
    tflops = flops / (ms / 1e3) / 1e12
    fp32_nominal = 148 * 128 * 2 * 1965e6 / 1e12
    if tf32:
        # dense TF32 tensor peak: half the measured bf16 GEMM peak (no TF32 figure is measured here)
        roof = {"bound": "tensor (TF32 projections) + fp32 SIMT attention", "achieved": tflops,
                "peak": peaks["bf16"] / 2, "unit": "TFLOP/s", "frac": tflops / (peaks["bf16"] / 2),
                "peak_source": f"half the {peaks['kind']} bf16 GEMM peak"}
    else:
        roof = {"bound": "fp32 FFMA (SIMT GEMMs)", "achieved": tflops, "peak": fp32_nominal, "unit": "TFLOP/s",
                "frac": tflops / fp32_nominal, "peak_source": "nominal: 148 SMs x 128 FFMA lanes x 2 x 1965 MHz"}
    o = O.Oracle(path, num_heads=H)
    x = seqs[0]
    tc = time.perf_counter()
    o.train_step(x[:cpu_tokens], x[1:cpu_tokens + 1], lr)
    cpu_s = time.perf_counter() - tc
    o.close()
    return {"metric": f"training tokens/sec (d={D}, one {M}-token sequence per step)", "value": M / (ms / 1e3),
            "unit": "tokens/s", "ms_per_step": ms, "steps": steps, "warmup": warmup,
            "e2e": {"value": M * steps / wall, "unit": "tokens/s", "h2d_bytes_per_step": 2 * 4 * M,
                    "d2h_bytes_per_step": 4, "api": "cortex_train_step (host token arrays, loss returned)"},
            "losses": losses, "dtype": "tf32 projections, fp32 otherwise" if tf32 else "fp32",
            "gpu_launches_total": launches, "flops_per_step": flops, "TFLOP/s": tflops, "roofline": roof,
            "config": {"workload": f"{c['model']}, V={V}, ctx {CTX}: cortex_train_step on {M} random ids per step",
                       "lr": lr},
            "cpu_baseline": {"value": cpu_tokens / cpu_s, "unit": "tokens/s", "cores": 1, "kind": "port",
                             "sample": f"the oracle's training step on the first {cpu_tokens} tokens ({cpu_s:.1f} s)"}}


def group_load_line(name, n, single_s):
    """Loads the configuration's model onto devices 0..n-1 from one process
    (cortex_group_load, one sequence slot per GPU) and reports the wall time
    beside a single-GPU load (cortex_load_stream_ex) of the same file."""
    import torch
    from snai_b200 import PREC_BF16, Cortex, CortexGroup
    c = CONFIGS[name]
    if torch.cuda.device_count() < n:
        return {"error": f"rank 0 sees {torch.cuda.device_count()} GPUs, fewer than {n}"}
    path = make_model(name)
    try:
        for i in range(n):  # every GPU's context exists before the timed loads
            torch.zeros(1, device=f"cuda:{i}")
            torch.cuda.synchronize(i)
        t0 = time.perf_counter()
        e = Cortex(path, num_heads=c["HEADS"], max_seqs=1, device=0, precision=PREC_BF16)
        one_s = time.perf_counter() - t0
        e.close()
        g = CortexGroup(path, c["HEADS"], n, list(range(n)), precision=PREC_BF16)
        out = {"devices": n, "seconds": g.load_seconds, "single_gpu_seconds": one_s,
               "rank_single_gpu_seconds": single_s, "model_bytes": os.path.getsize(path),
               "how": "one file read into GPU 0 (pinned double-buffered), peer copies to the others, bf16 packing "
                      "on every GPU"}
        # the federated average of the n engines' weights (cortex_group_average):
        # each GPU reads its shard from every GPU (peer loads), then copies the
        # other shards in (peer copies); NVLink bytes per GPU, each way
        g.average()
        t0 = time.perf_counter()
        reps = 5
        for _ in range(reps):
            g.average()
        avg_s = (time.perf_counter() - t0) / reps
        wbytes = (os.path.getsize(path) - 28)
        link = 2.0 * wbytes * (n - 1) / n
        out["average"] = {"seconds": avg_s, "weight_bytes": wbytes, "nvlink_bytes_per_gpu": link,
                          "GB/s_per_gpu": link / avg_s / 1e9, "peer_copy_reference_GB/s": 770.0,
                          "timing": f"wall clock over {reps} calls, each waiting for every GPU"}
        g.close()
        return out
    except Exception as ex:  # noqa: BLE001
        return {"error": f"{type(ex).__name__}: {ex}"}


def tokenizer_bench(vocab_path, n_words=200000):
    """Encode/decode throughput of the library's C++ tokenizer
    (cortex_tokenizer_*) on seeded text (words of the vocabulary joined by
    spaces and newlines), beside the oracle's Python restatement of
    src/snai_tokenizer.php on a tenth of it.  Host code: no GPU involved."""
    import ctypes

    import oracle.tokenizer as OT
    from snai_b200 import load
    lib = load()
    ot = OT.Tokenizer(vocab_path)
    rng = np.random.default_rng(5)
    words = [w.replace(OT.META, "") for w in ot.vocab if w.startswith(OT.META) and len(w) > 1][:4000] or ["abc"]
    pick = rng.integers(0, len(words), n_words)
    text = "".join(words[i] + ("\n" if k % 17 == 16 else " ") for k, i in enumerate(pick)).encode("utf-8")
    h = lib.cortex_tokenizer_load(vocab_path.encode())
    n = lib.cortex_tokenizer_encode(h, text, len(text), None, 0)  # warms the merge cache
    ids = np.zeros(n, dtype=np.int32)
    t0 = time.perf_counter()
    lib.cortex_tokenizer_encode(h, text, len(text), ids.ctypes.data_as(ctypes.c_void_p), n)
    enc_s = time.perf_counter() - t0
    buf = ctypes.create_string_buffer(len(text) * 2 + 16)
    t0 = time.perf_counter()
    lib.cortex_tokenizer_decode(h, ids.ctypes.data_as(ctypes.c_void_p), n, 0, buf, len(buf))
    dec_s = time.perf_counter() - t0
    lib.cortex_tokenizer_free(h)
    sub_text = text[:len(text) // 10].decode("utf-8", errors="ignore")
    ot.encode(sub_text)
    t0 = time.perf_counter()
    py_ids = ot.encode(sub_text)
    py_s = time.perf_counter() - t0
    return {"metric": "tokenizer encode MB/s (host)", "value": len(text) / enc_s / 1e6, "unit": "MB/s",
            "tokens_per_s": n / enc_s, "decode_tokens_per_s": n / dec_s, "bytes": len(text), "tokens": n,
            "cpu_baseline": {"value": len(sub_text.encode()) / py_s / 1e6, "unit": "MB/s", "cores": 1, "kind": "port",
                             "sample": f"oracle/tokenizer.py (Python restatement of the PHP encode) on "
                                       f"{len(py_ids)} tokens"},
            "vocab": os.path.basename(vocab_path)}


def gemm_bench(args):
    """Projection micro-benchmark: the d=1024 decode step's GEMM shapes
    (`--seqs` rows; qkv N=3072, wo N=1024, up N=4096, down N=1024 with
    K=4096, logits N=16384) through decode passes of one token per slot, on
    the benchmark model's weights at positions 16..  One JSON line per GEMM
    kind: TFLOP/s from the library's CUDA-event profiler against the measured
    bf16 peak (BF16 mode); below 64 rows the engine runs in FP32 mode, whose
    projections are fp32 GEMVs, and the line gives GB/s against the measured
    copy peak."""
    import torch
    from snai_b200 import PREC_BF16, PREC_FP32, Cortex
    peaks = load_peaks()
    B = args.seqs
    eng = Cortex(make_model("c4"), num_heads=16, max_seqs=B, precision=PREC_FP32 if B < 64 else PREC_BF16)
    dev = torch.device("cuda")
    rng = np.random.default_rng(7)
    stream = torch.cuda.Stream(device=dev)
    eng.set_stream(stream.cuda_stream)
    torch.cuda.set_stream(stream)
    eng.forward_dev(torch.from_numpy(rng.integers(0, V, 16 * B).astype(np.int32)).to(dev), B, 16)

    def step():
        if eng.pos(0) >= 48:
            eng.rewind(16)
        toks = torch.from_numpy(rng.integers(0, V, B).astype(np.int32)).to(dev)
        if B < 64:
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
    for k in ("qkv", "wo", "up", "down", "logits"):
        n, ms, nbytes, flops = prof[k]
        if not n:
            continue
        tf = flops / (ms / 1e3) / 1e12
        if B < 64:
            gbs = nbytes / (ms / 1e3) / 1e9
            print(json.dumps({"metric": "projection GB/s (fp32 GEMV)", "gemm": k, "value": gbs, "unit": "GB/s",
                              "rows": B, "launches": n, "us_per_launch": 1e3 * ms / n,
                              "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm"], "unit": "GB/s",
                                           "frac": gbs / peaks["hbm"]}}), flush=True)
            continue
        print(json.dumps({"metric": "projection TFLOP/s", "gemm": k, "value": tf, "unit": "TFLOP/s", "rows": B,
                          "launches": n, "us_per_launch": 1e3 * ms / n,
                          "roofline": {"bound": "tensor", "achieved": tf, "peak": peaks["bf16"], "unit": "TFLOP/s",
                                       "frac": tf / peaks["bf16"],
                                       "frac_sustained": tf / peaks["bf16_sustained"]}}), flush=True)
    eng.close()


def our_arm(args, rank, world, local_rank):
    import torch
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist_ = Dist(world, dev)
    peaks = load_peaks()
    c = CONFIGS[args.config]
    res = decode_run(args.config, args, rank, world, local_rank, dist_, peaks)
    if rank == 0:
        line = {"metric": res["metric"], "value": res["value"], "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": res["ms_per_step"],
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (seeded model, random prompt ids, seeded uniforms)", "config": config_dict(c)}
        for k in ("e2e", "gpu_launches", "roofline", "positions", "kernels", "ids_sha256", "prefill", "load_s",
                  "clocks"):
            line[k] = res[k]
        if world == 1 and not args.no_cpu_baseline:
            nthreads = os.cpu_count() or 1
            start, p0 = window(c, args.steps, args.warmup)
            n_cpu = min(args.steps, 2)
            rate, secs, nseq = cpu_sample(args.config, n_cpu, nthreads, p0)
            line["cpu_baseline"] = {"value": rate, "unit": "tokens/s", "cores": nthreads, "kind": "port",
                                    "sample": f"{nseq} sequences x {n_cpu} decode steps from position {p0}, one "
                                              f"thread per sequence ({secs:.1f} s)"}
    if world > 1 and not args.no_extras:
        # one process loading the model onto every GPU of the run: one file
        # read, fp32 weights fanned out from the first GPU by peer copies
        # (cortex_group_load), beside this rank's own single-GPU load
        dist_.barrier()
        if rank == 0:
            line["group_load"] = group_load_line(args.config, world, res["load_s"])
        dist_.barrier()
    if world == 1 and args.config == "c4" and not args.no_extras:
        # the other workloads of the metric, one GPU; a failure is recorded
        # in its key and does not lose the headline line
        for name in ("c3", "c2"):
            try:
                r = decode_run(name, args, 0, 1, local_rank, dist_, peaks, extra=True)
                line[name] = {k: r[k] for k in ("metric", "value", "unit", "ms_per_step", "e2e", "roofline",
                                                "positions", "ids_sha256", "prefill", "clocks")}
                line[name]["config"] = config_dict(CONFIGS[name])
                line[name]["kernels"] = {k: {kk: vv for kk, vv in v.items()
                                             if kk in ("share", "GB/s", "TFLOP/s", "frac_hbm", "frac_bf16_sustained")}
                                         for k, v in r["kernels"].items()}
            except Exception as ex:  # noqa: BLE001
                line[name] = {"error": f"{type(ex).__name__}: {ex}"}
        for key, fn in (("gemv_pass", gemv_pass_line),
                        ("gemv_pass_persistent", lambda p: gemv_pass_line(p, fused=True)),
                        ("gemv_pass_pos1000", lambda p: gemv_pass_line(p, pos=1000)),
                        ("gemv_pass_pos1000_unsplit", lambda p: gemv_pass_line(p, pos=1000, split=False)),
                        ("sampling", sampling_lines),
                        ("train_c2", lambda p: train_line(p, "c2")),
                        ("train_c4", lambda p: train_line(p, "c4")),
                        ("train_c4_tf32", lambda p: train_line(p, "c4", tf32=True))):
            try:
                line[key] = fn(peaks)
            except Exception as ex:  # noqa: BLE001
                line[key] = {"error": f"{type(ex).__name__}: {ex}"}
    if rank == 0:
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20, help="timed decode steps (512: the whole generation)")
    ap.add_argument("--config", choices=["c4", "c3", "c2"], default="c4",
                    help="c4 (default): the headline d=1024 workload; c3 / c2: the smaller configurations alone")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the c3/c2/sampling/GEMV extra keys")
    ap.add_argument("--sampler", action="store_true", help="only the isolated sampling workload, one line each")
    ap.add_argument("--gemm", action="store_true", help="only the projection micro-benchmark")
    ap.add_argument("--tokenizer", metavar="VOCAB_JSON", help="only the tokenizer throughput (host code)")
    ap.add_argument("--train", action="store_true", help="only the training-step lines (c2 and c4 models)")
    ap.add_argument("--pass-lines", action="store_true",
                    help="only the one-row fp32 pass lines (kernel per stage, persistent kernel, position 1000)")
    ap.add_argument("--seqs", type=int, default=None,
                    help="total sequences of the decode configuration (default: the configuration's), or rows of "
                         "the projection micro-benchmark (default 4096)")
    args = ap.parse_args()
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
    if args.tokenizer:
        print(json.dumps(tokenizer_bench(args.tokenizer)), flush=True)
        return
    if args.pass_lines:
        if rank == 0:
            p = load_peaks()
            for key, kw in (("gemv_pass", {}), ("gemv_pass_persistent", {"fused": True}),
                            ("gemv_pass_pos1000", {"pos": 1000})):
                print(json.dumps(dict(key=key, **gemv_pass_line(p, **kw))), flush=True)
        return
    if args.train:
        if rank == 0:
            for name, tf32 in (("c2", False), ("c4", False), ("c2", True), ("c4", True)):
                print(json.dumps(train_line(load_peaks(), name, steps=args.steps, warmup=args.warmup, tf32=tf32)),
                      flush=True)
        return
    if args.gemm:
        if args.seqs is None:
            args.seqs = 4096
        if rank == 0:
            gemm_bench(args)
        return
    if args.seqs is not None:
        CONFIGS[args.config] = dict(CONFIGS[args.config], SEQS=args.seqs)
    if args.sampler:
        if rank == 0:
            for ln in sampling_lines(load_peaks(), steps=args.steps, warmup=args.warmup):
                print(json.dumps(dict(metric="sampling GB/s", **ln)), flush=True)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        our_arm(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
