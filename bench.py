"""Benchmark: the ACT policy step on N B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One policy replica per GPU (requests are independent: "replicas only", no
collective in the step loop). Each timed step is one captured CUDA graph
(frame normalize -> int8 ResNet-18 -> token assembly -> 4 encoder layers ->
decoder -> head) on device-resident inputs, timed with CUDA events on the
launching stream; L2 is flushed (256 MiB memset, outside the events) between
steps. `value` = chunks/s of the whole job = N*K / max over ranks of the summed
step time. `e2e` = the same metric through the C ABI (vla_act_predict) with
pinned host frames/state in and host actions out, copies included, wall clock.

Extra fields: per-step latency p50/p95, the W8A8 GEMM alone at the ACT FFN
shape (602x3200x512; TOPS cold and L2-warm) as the
roofline of the dominant kernel, the reference's own CPU implementation timed
on this host as `cpu_baseline`, and SM clocks sampled during the timed region.

--impl reference times the reference's CPU implementation (oracle/_ref, the
reference's unmodified sources built here; all host threads) on the same
workload and prints the same JSON line with "impl": "reference".
"""
from __future__ import annotations

import argparse
import ctypes
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

METRIC = "ACT policy throughput (chunks/s, bs1 per replica); p50 chunk latency; int8 GEMM TOPS"
INT8_MASK = 63
GEMM_SHAPE = (602, 3200, 512)          # ACT encoder FFN w1: M x N x K
GEMM_OPS = 2 * 602 * 3200 * 512        # 1,972,633,600 int8 ops per call
# compulsory bytes of one dense_linear_i8 call: x fp32 + W int8 + out fp32 + scales/bias
GEMM_BYTES = 602 * 512 * 4 + 3200 * 512 + 602 * 3200 * 4 + 3200 * 8 + 602 * 4


def _env_rank():
    return int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0")), \
        int(os.environ.get("WORLD_SIZE", "1"))


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("bf16_tflops", 1590.0), d.get("hbm_gbs", 6650.0), "measured"
    return 1590.0, 6650.0, "fallback"


def _traffic():
    """dram bytes per GEMM launch from the committed ncu summary (profiles/), if any."""
    p = os.path.join(ROOT, "profiles", "gemm_ffn_traffic.json")
    if os.path.exists(p):
        try:
            return json.load(open(p)).get("dram_bytes_per_launch")
        except Exception:
            return None
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.f = None

    def __enter__(self):
        try:
            self.f = tempfile.TemporaryFile(mode="w+")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.f:
            return None
        self.f.seek(0)
        sms, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.f.read().strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sms.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sms:
            return None
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sms)}


def max_over_ranks(seconds: float, dist=None, device=None) -> float:
    """The job's time for a timed region: the slowest rank's (max-reduce), or
    the local time on one process. Runs outside the timed region."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return seconds
    import torch
    t = torch.tensor([seconds], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def job_value(steps_per_rank: int, world: int, seconds_max: float) -> float:
    """Whole-job chunks/s: every rank's steps over the slowest rank's time."""
    return world * steps_per_rank / seconds_max


_PINNED = []   # page-locked tensors behind the numpy views pinned() hands out


def pinned(torch, a):
    """A copy of the numpy array `a` in page-locked host memory: the e2e legs
    feed the C ABI from pinned buffers, as a serving loop that owns its camera
    buffers does (the copies stay inside the timed region)."""
    a = np.ascontiguousarray(a)
    t = torch.empty(a.shape, dtype=torch.from_numpy(a).dtype, pin_memory=True)
    _PINNED.append(t)
    out = t.numpy()
    out[...] = a
    return out


def timed_calls(fn, n: int):
    """Wall-clock seconds of each of n calls of fn(i)."""
    out = []
    for i in range(n):
        t0 = time.perf_counter()
        fn(i)
        out.append(time.perf_counter() - t0)
    return out


def cpu_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_model():
    """The host CPU as lscpu names it: model name, physical cores (core ids per
    socket), logical CPUs this process may use."""
    model, cores = None, set()
    try:
        phys = None
        with open("/proc/cpuinfo") as f:
            for line in f:
                k, _, v = line.partition(":")
                k, v = k.strip(), v.strip()
                if k == "model name" and model is None:
                    model = v
                elif k == "physical id":
                    phys = v
                elif k == "core id":
                    cores.add((phys, v))
    except OSError:
        pass
    return {"model": model or "unknown", "physical_cores": len(cores) or None, "logical_cpus": cpu_cores()}


# ----------------------------------------------------------------- CPU side

_CPU_CHILD = r"""
import json, os, sys, time
sys.path.insert(0, %(root)r)
import numpy as np
from vla_simd_b200 import synth
kind, budget, max_steps, warmup = %(kind)r, %(budget)f, %(max_steps)d, %(warmup)d
f, s = synth.act_inputs(synth.ACT_BASELINE, seed=1)
from oracle import oracle
r = oracle.reference()
if r is None:
    print(json.dumps({"unavailable": "oracle/_ref/libvla_ref.so (the reference's own build) not present"}))
    sys.exit(0)
l = r.l
h = l.vla_act_load(%(ckpt)r.encode())
out = np.zeros((100, 6), np.float32)
P = lambda a: a.ctypes.data_as(__import__("ctypes").c_void_p)
for _ in range(warmup):
    l.vla_act_predict(h, P(f), P(s), 1, P(out))
times = []
t_end = time.perf_counter() + budget
while len(times) < max_steps and (not times or time.perf_counter() < t_end):
    t0 = time.perf_counter()
    rc = l.vla_act_predict(h, P(f), P(s), 1, P(out))
    times.append(time.perf_counter() - t0)
    assert rc == 0
l.vla_act_free(h)
print(json.dumps({"steps": len(times), "seconds": sum(times), "p50_ms": 1e3 * float(np.median(times))}))
"""


def time_reference_cpu(ckpt: str, budget_s: float, max_steps: int, threads: int | None = None, warmup: int = 3):
    """The reference's own ACT step (oracle/_ref) in a fresh process with all host cores (or `threads`),
    after `warmup` untimed steps."""
    cores = threads or cpu_cores()
    env = dict(os.environ, ACT_INT8=str(INT8_MASK), OMP_NUM_THREADS=str(cores), OMP_PROC_BIND="close",
               CUDA_VISIBLE_DEVICES="")
    code = _CPU_CHILD % {"root": ROOT, "kind": "reference", "budget": budget_s, "max_steps": max_steps,
                         "ckpt": ckpt, "warmup": warmup}
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=900)
    if r.returncode != 0:
        return {"unavailable": f"reference CPU run failed: {r.stderr.strip().splitlines()[-1:]}"}
    d = json.loads(r.stdout.strip().splitlines()[-1])
    if "unavailable" in d:
        return d
    d["cores"] = cores
    d["chunks_per_s"] = d["steps"] / d["seconds"]
    return d


# ----------------------------------------------------------------- GPU side

def time_gemm(torch, dev, n_cold=30, n_warm_graph=50, n_lin=10):
    """The dominant op alone: quantize + tcgen05 W8A8 GEMM at the ACT FFN shape."""
    from vla_simd_b200 import ops
    M, N, K = GEMM_SHAPE
    rng = np.random.default_rng(0)
    x = torch.from_numpy(rng.standard_normal((M, K), dtype=np.float32)).to(dev)
    W = torch.from_numpy((rng.standard_normal((N, K), dtype=np.float32) * 0.02).astype(np.float32)).to(dev)
    b = torch.from_numpy((rng.standard_normal(N, dtype=np.float32) * 0.01).astype(np.float32)).to(dev)
    wq, ws = ops.pack_weights_i8(W)
    xq, xs = ops.quantize_act_i8(x)
    out = torch.empty((M, N), device=dev)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    st = torch.cuda.current_stream()

    def gemm():
        ops.gemm_i8(xq, xs, wq, ws, K, bias=b, out=out)

    for _ in range(3):
        gemm()
    # cold: L2 flushed before each launch
    cold = []
    for _ in range(n_cold):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        gemm()
        e1.record(st)
        e1.synchronize()
        cold.append(e0.elapsed_time(e1) * 1e-3)
    # L2-warm: back-to-back launches captured in one graph
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(n_warm_graph):
            gemm()
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(2):
        g.replay()
    e1.record(st)
    e1.synchronize()
    warm = e0.elapsed_time(e1) * 1e-3 / (2 * n_warm_graph)
    # fused quantize + GEMM (dense_linear_i8 entry point), cold
    lin = []
    for _ in range(n_lin):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        ops.dense_linear_i8(x, wq, ws, b)
        e1.record(st)
        e1.synchronize()
        lin.append(e0.elapsed_time(e1) * 1e-3)
    del g
    tc = statistics.median(cold)
    return {"shape": "602x3200x512 (M x N x K)", "us_cold": tc * 1e6, "us_l2_warm": warm * 1e6,
            "tops_cold": GEMM_OPS / tc / 1e12, "tops_l2_warm": GEMM_OPS / warm / 1e12,
            "dense_linear_i8_us_cold": statistics.median(lin) * 1e6}


def run_gemm_msweep():
    """The W8A8 GEMM at the FFN shape for M = 602 x {1, 8, 32, 128} (batched
    policies), back-to-back launches in a CUDA graph. Per M: time per call,
    int8 TOPS against the measured tensor peak, and the compulsory-bytes
    roofline (int8 A and W, fp32 out, scales) against measured HBM bandwidth."""
    import torch
    from vla_simd_b200 import ops
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    N, K = GEMM_SHAPE[1], GEMM_SHAPE[2]
    bf16_peak, hbm, peak_kind = _peaks()
    peak_tops = 2.0 * bf16_peak
    st = torch.cuda.Stream()
    for mult in (1, 8, 32, 128):
        M = GEMM_SHAPE[0] * mult
        g = torch.Generator(device="cpu").manual_seed(M)
        xq = torch.randint(-127, 128, (M, K), dtype=torch.int8, generator=g).to(dev)
        wq = torch.randint(-127, 128, (N, K), dtype=torch.int8, generator=g).to(dev)
        xs, ws = torch.rand(M, device=dev) * 1e-3, torch.rand(N, device=dev) * 1e-3
        b, out = torch.rand(N, device=dev), torch.empty(M, N, device=dev)
        with torch.cuda.stream(st):
            ops.gemm_i8(xq, xs, wq, ws, K, bias=b, out=out)
        torch.cuda.synchronize()
        reps = max(4, 200 // mult)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=st):
            for _ in range(reps):
                ops.gemm_i8(xq, xs, wq, ws, K, bias=b, out=out)
        ts = []
        for r in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(st):
                e0.record(st)
                gr.replay()
                e1.record(st)
            torch.cuda.synchronize()
            if r:
                ts.append(e0.elapsed_time(e1) * 1e-3 / reps)
        del gr
        t = statistics.median(ts)
        ops_ = 2.0 * M * N * K
        nbytes = M * K + N * K + 4.0 * M * N + 4.0 * (M + 2 * N)
        print(json.dumps({"op": "gemm_i8", "M": M, "N": N, "K": K, "us_per_call": round(t * 1e6, 2),
                          "tops": round(ops_ / t / 1e12, 1), "tensor_frac": round(ops_ / t / 1e12 / peak_tops, 4),
                          "hbm_gbs_compulsory": round(nbytes / t / 1e9, 1), "hbm_frac": round(nbytes / t / 1e9 / hbm, 4),
                          "peak_source": peak_kind}), flush=True)


def run_op(name: str, iters: int = 20):
    """One op at its ACT-step shape, timed alone (also the small cases ncu captures use)."""
    import torch
    from vla_simd_b200 import EPI_ADD, EPI_RELU, ops
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    g = torch.Generator(device="cpu").manual_seed(0)
    rnd = lambda *sh, s=1.0: (torch.randn(*sh, generator=g) * s).to(dev)  # noqa: E731
    T, d, ff = 602, 512, 3200
    if name == "gemm_msweep":
        return run_gemm_msweep()
    if name == "attention":
        qk, v = rnd(T, 2 * d), rnd(T, d)
        fn = lambda: ops.gqa_attention(qk[:, :d], qk[:, d:], v, 8, 8, 0.125)  # noqa: E731
        work = 4 * 8 * T * T * 64
    elif name in ("gemm_qkv", "gemm_w1", "gemm_w2"):
        M, N, K, mode = {"gemm_qkv": (T, 512, d, 0), "gemm_w1": (T, ff, d, EPI_RELU),
                         "gemm_w2": (T, d, ff, EPI_ADD)}[name]
        wq, ws = ops.pack_weights_i8(rnd(N, K, s=0.02))
        xq, xs = ops.quantize_act_i8(rnd(M, K))
        b, res = rnd(N), rnd(M, N)
        fn = lambda: ops.gemm_i8(xq, xs, wq, ws, K, bias=b, mode=mode, res=res if mode == EPI_ADD else None)  # noqa
        work = 2 * M * N * K
    elif name == "layernorm":
        x, w, b = rnd(T, d), rnd(d), rnd(d)
        fn = lambda: ops.layernorm(x, w, b)  # noqa: E731
        work = 2 * T * d * 4
    elif name == "quantize":
        x = rnd(T, ff)
        fn = lambda: ops.quantize_act_i8(x)  # noqa: E731
        work = T * ff * 5
    elif name == "conv_layer1":
        x = rnd(2, 120, 160, 64)
        wq, ws = ops.pack_weights_i8(rnd(64, 9 * 64, s=0.05))
        b = rnd(64)
        fn = lambda: ops.conv2d_i8(x, wq, ws, b, 64, 3, 1, 1, mode=EPI_RELU)  # noqa: E731
        work = 2 * 2 * 120 * 160 * 64 * 576
    else:
        raise SystemExit(f"unknown --op {name}")
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / iters
    print(json.dumps({"op": name, "us_per_call": round(us, 3), "work_per_call": work,
                      "rate_per_s": work / us * 1e6}), flush=True)


def run_ours(args):
    import torch
    rank, local_rank, world = _env_rank()
    os.environ["VLA_CUDA_DEVICE"] = str(local_rank)
    os.environ["ACT_INT8"] = str(INT8_MASK)
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    from vla_simd_b200 import ActPolicy, synth

    ckpt_root = tempfile.mkdtemp(prefix="vla_act_")
    ckpt = synth.write_act_checkpoint(os.path.join(ckpt_root, "act"), synth.ACT_BASELINE, seed=0)
    pol = ActPolicy(ckpt)
    frames, state = synth.act_inputs(synth.ACT_BASELINE, seed=1 + rank)
    # one C-ABI call leaves this observation resident in the policy's device
    # input buffers; the timed steps then run on device-resident inputs
    pol.predict(frames, state)
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(device=dev)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    for _ in range(max(args.warmup, 3)):
        pol.enqueue(stream.cuda_stream)
    torch.cuda.synchronize()
    kernels = pol.kernels_per_step

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        for i in range(args.steps):
            with torch.cuda.stream(stream):
                flush.zero_()
            starts[i].record(stream)
            pol.enqueue(stream.cuda_stream)
            ends[i].record(stream)
        torch.cuda.synchronize()
    if dist:
        dist.barrier()
    step_s = [s.elapsed_time(e) * 1e-3 for s, e in zip(starts, ends)]
    total_max = max_over_ranks(sum(step_s), dist, dev)
    value = job_value(args.steps, world, total_max)

    # e2e through the C ABI with host buffers (copies inside), wall clock
    n_e2e = max(args.steps, 10)
    frames_h, state_h = pinned(torch, frames), pinned(torch, state)
    for _ in range(3):
        pol.predict(frames_h, state_h)
    if dist:
        dist.barrier()
    calls = timed_calls(lambda i: pol.predict(frames_h, state_h), n_e2e)
    e2e_s = max_over_ranks(sum(calls), dist, dev)
    e2e = {"value": job_value(n_e2e, world, e2e_s), "unit": "chunks/s", "h2d_bytes_per_step": frames.nbytes + state.nbytes,
           "d2h_bytes_per_step": 100 * 6 * 4, "p50_ms_per_call": 1e3 * statistics.median(calls),
           "path": "vla_act_predict (C ABI), pinned host uint8 frames + state -> host actions"}

    gemm = time_gemm(torch, dev) if rank == 0 else None
    cpu = cpu1 = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:   # the CPU baseline runs at N=1 only
        cpu = time_reference_cpu(ckpt, budget_s=args.cpu_budget, max_steps=40)
        cpu1 = time_reference_cpu(ckpt, budget_s=min(args.cpu_budget, 8.0), max_steps=12, threads=1)
    pol.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    bf16_peak, hbm_peak, peak_kind = _peaks()
    int8_peak = 2.0 * bf16_peak   # dense int8 runs at 2x the dense bf16 rate on B200
    achieved = gemm["tops_l2_warm"]
    roofline = {"kernel": "w8a8_slab_kernel<128, 128> (ACT FFN 602x3200x512, L2-warm, back-to-back)", "bound": "tensor",
                "achieved": round(achieved, 2), "peak": round(int8_peak, 1), "unit": "TOPS (int8)",
                "frac": round(achieved / int8_peak, 4),
                "peak_note": f"2x {peak_kind} bf16 dense ({bf16_peak} TFLOP/s, MEASURED_PEAKS.json)",
                "traffic": _traffic(),
                "cold": {"achieved_tops": round(gemm["tops_cold"], 2),
                         "hbm_bound_us": round(GEMM_BYTES / (hbm_peak * 1e9) * 1e6, 3),
                         "us": round(gemm["us_cold"], 3)}}
    cpu_baseline = None
    if cpu and "unavailable" not in cpu:
        cpu_baseline = {"value": round(cpu["chunks_per_s"], 3), "unit": "chunks/s", "cores": cpu["cores"],
                        "kind": "reference", "p50_ms": round(cpu["p50_ms"], 2),
                        "sample": f"{cpu['steps']} ACT steps (same checkpoint, ACT_INT8=63) of the reference's "
                                  f"own vla_act_predict, OMP_NUM_THREADS={cpu['cores']}, OMP_PROC_BIND=close",
                        "cpu": cpu_model()}
        if cpu1 and "unavailable" not in cpu1:
            cpu_baseline["one_thread"] = {"value": round(cpu1["chunks_per_s"], 3), "p50_ms": round(cpu1["p50_ms"], 2),
                                          "steps": cpu1["steps"], "sample": "OMP_NUM_THREADS=1"}
    elif cpu:
        cpu_baseline = {"unavailable": cpu["unavailable"]}
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "chunks/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": round(1e3 * total_max / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8 (W8A8 GEMMs, int32 acc) + fp32",
        "data": "synthetic (seeded random-init ACT weights, uniform uint8 frames, N(0,1) state)",
        "config": {"workload": "ACT policy step, BASELINE configs[1]: 2x480x640 uint8 frames -> ResNet-18 -> "
                               "602-token 4-layer encoder, 1-layer decoder, 100x6 actions; bs1 per GPU",
                   "int8_mask": INT8_MASK, "parallelism": f"replicas x{world} (no collective)",
                   "l2": "flushed between steps (256 MiB memset outside the timed events)"},
        "latency_ms": {"p50": round(1e3 * statistics.median(step_s), 4),
                       "p95": round(1e3 * float(np.percentile(step_s, 95)), 4)},
        "int8_gemm": {k: (round(v, 3) if isinstance(v, float) else v) for k, v in gemm.items()},
        "roofline": roofline, "cpu_baseline": cpu_baseline, "e2e": e2e,
        "gpu_launches": kernels * args.steps, "kernels_per_step": kernels,
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


_DP_CPU_CHILD = r"""
import ctypes, json, os, sys, time
sys.path.insert(0, %(root)r)
import numpy as np
from vla_simd_b200 import synth
budget, max_steps = %(budget)f, %(max_steps)d
f, s, n = synth.dp_inputs(synth.DP_BASELINE, seed=1)
from oracle import oracle
r = oracle.reference()
if r is None:
    print(json.dumps({"unavailable": "oracle/_ref/libvla_ref.so (the reference's own build) not present"}))
    sys.exit(0)
l = r.l
l.vla_diffusion_load.restype = ctypes.c_void_p
l.vla_diffusion_load.argtypes = [ctypes.c_char_p]
l.vla_diffusion_predict.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int32] + [ctypes.c_void_p] * 2
l.vla_diffusion_free.argtypes = [ctypes.c_void_p]
h = l.vla_diffusion_load(%(ckpt)r.encode())
out = np.zeros((synth.DP_BASELINE.n_action_steps, synth.DP_BASELINE.action_dim), np.float32)
P = lambda a: a.ctypes.data_as(ctypes.c_void_p)
l.vla_diffusion_predict(h, P(f), P(s), 1, P(out), P(n))
times = []
t_end = time.perf_counter() + budget
while len(times) < max_steps and (not times or time.perf_counter() < t_end):
    t0 = time.perf_counter()
    rc = l.vla_diffusion_predict(h, P(f), P(s), 1, P(out), P(n))
    times.append(time.perf_counter() - t0)
    assert rc == 0
l.vla_diffusion_free(h)
print(json.dumps({"steps": len(times), "seconds": sum(times), "p50_ms": 1e3 * float(np.median(times))}))
"""

DP_MASK = 3   # DIFFUSION_INT8: U-Net GEMMs and backbone convs in W8A8


def time_reference_dp_cpu(ckpt: str, budget_s: float, max_steps: int):
    """The reference's own Diffusion Policy query (oracle/_ref) in a fresh process, all host cores."""
    cores = cpu_cores()
    env = dict(os.environ, DIFFUSION_INT8=str(DP_MASK), OMP_NUM_THREADS=str(cores), OMP_PROC_BIND="close",
               CUDA_VISIBLE_DEVICES="")
    code = _DP_CPU_CHILD % {"root": ROOT, "budget": budget_s, "max_steps": max_steps, "ckpt": ckpt}
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=900)
    if r.returncode != 0:
        return {"unavailable": f"reference CPU run failed: {r.stderr.strip().splitlines()[-1:]}"}
    d = json.loads(r.stdout.strip().splitlines()[-1])
    if "unavailable" in d:
        return d
    d["cores"] = cores
    d["chunks_per_s"] = d["steps"] / d["seconds"]
    return d


def run_dp(args):
    """Diffusion Policy: one query batch per step, every
    query its own observation history and noise, DDIM 10; replicas per GPU."""
    import torch
    rank, local_rank, world = _env_rank()
    os.environ["VLA_CUDA_DEVICE"] = str(local_rank)
    os.environ["DIFFUSION_INT8"] = str(DP_MASK)
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    from vla_simd_b200 import DiffusionPolicy, synth
    B = args.batch
    ckpt_root = tempfile.mkdtemp(prefix="vla_dp_")
    ckpt = synth.write_dp_checkpoint(os.path.join(ckpt_root, "dp"), synth.DP_BASELINE, seed=0)
    pol = DiffusionPolicy(ckpt, max_batch=B)
    frames, state, noise = synth.dp_inputs(synth.DP_BASELINE, seed=1 + rank, batch=B)
    pol.predict_batch(frames, state, noise)   # leaves the batch resident in the device input buffers
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(device=dev)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    for _ in range(max(args.warmup, 3)):
        pol.enqueue(B, stream.cuda_stream)
    torch.cuda.synchronize()
    kernels = pol.kernels_per_step
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        for i in range(args.steps):
            with torch.cuda.stream(stream):
                flush.zero_()
            starts[i].record(stream)
            pol.enqueue(B, stream.cuda_stream)
            ends[i].record(stream)
        torch.cuda.synchronize()
    if dist:
        dist.barrier()
    step_s = [s_.elapsed_time(e_) * 1e-3 for s_, e_ in zip(starts, ends)]
    total_max = max_over_ranks(sum(step_s), dist, dev)
    value = job_value(args.steps * B, world, total_max)
    n_e2e = max(args.steps, 10)
    frames_h, state_h, noise_h = pinned(torch, frames), pinned(torch, state), pinned(torch, noise)
    for _ in range(2):
        pol.predict_batch(frames_h, state_h, noise_h)
    if dist:
        dist.barrier()
    calls = timed_calls(lambda i: pol.predict_batch(frames_h, state_h, noise_h), n_e2e)
    e2e_s = max_over_ranks(sum(calls), dist, dev)
    e2e = {"value": job_value(n_e2e * B, world, e2e_s), "unit": "chunks/s",
           "h2d_bytes_per_step": frames.nbytes + state.nbytes + noise.nbytes,
           "d2h_bytes_per_step": B * pol.chunk * pol.action_dim * 4, "p50_ms_per_call": 1e3 * statistics.median(calls),
           "path": "vla_diffusion_predict_batch (C ABI), pinned host frames + state + noise -> host actions"}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:   # the CPU baseline runs at N=1 only
        cpu = time_reference_dp_cpu(ckpt, budget_s=args.cpu_budget, max_steps=20)
    pol.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    cpu_baseline = None
    if cpu and "unavailable" not in cpu:
        cpu_baseline = {"value": round(cpu["chunks_per_s"], 3), "unit": "chunks/s", "cores": cpu["cores"],
                        "kind": "reference", "p50_ms": round(cpu["p50_ms"], 2),
                        "sample": f"{cpu['steps']} single queries (same checkpoint, DIFFUSION_INT8={DP_MASK}) of "
                                  f"the reference's own vla_diffusion_predict, OMP_NUM_THREADS={cpu['cores']}"}
    elif cpu:
        cpu_baseline = {"unavailable": cpu["unavailable"]}
    print(json.dumps({
        "metric": "Diffusion Policy throughput (chunks/s)", "value": round(value, 3), "unit": "chunks/s",
        "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3),
        "ms_per_step": round(1e3 * total_max / args.steps, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8 (W8A8 GEMMs, int32 acc) + fp32",
        "data": "synthetic (seeded random-init DP weights, uniform uint8 frames, N(0,1) state and noise)",
        "config": {"workload": "Diffusion Policy, BASELINE configs[2]: 2-frame history of 96x96 frames "
                               "center-cropped to 84x84 -> ResNet-18 (GroupNorm) + spatial softmax; U-Net "
                               "(512, 1024, 2048) k5 GN8 FiLM, horizon 16, action 2, DDIM 10",
                   "batch_per_gpu": B, "int8_mask": DP_MASK, "parallelism": f"replicas x{world} (no collective)",
                   "l2": "flushed between steps (256 MiB memset outside the timed events)"},
        "latency_ms": {"p50": round(1e3 * statistics.median(step_s), 4),
                       "p95": round(1e3 * float(np.percentile(step_s, 95)), 4)},
        "cpu_baseline": cpu_baseline, "e2e": e2e, "gpu_launches": kernels * args.steps,
        "kernels_per_step": kernels, "clocks": clk.summary(),
    }), flush=True)


OCTO_MASK = 63   # OCTO_INT8: every transformer / projection / stem / head GEMM in W8A8

_OCTO_CPU_CHILD = r"""
import ctypes, json, os, sys, time
sys.path.insert(0, %(root)r)
import numpy as np
from vla_simd_b200 import synth
budget, max_steps = %(budget)f, %(max_steps)d
sh = synth.OCTO_BASELINE
rng = np.random.default_rng(11)
prim = rng.integers(0, 256, size=(max_steps + 2, 256, 256, 3), dtype=np.uint8)
wrist = rng.integers(0, 256, size=(max_steps + 2, 128, 128, 3), dtype=np.uint8)
tm = np.ones(sh.window, np.uint8)
ins = synth.octo_instruction(1)
from oracle import oracle
r = oracle.reference()
if r is None:
    print(json.dumps({"unavailable": "oracle/_ref/libvla_ref.so (the reference's own build) not present"}))
    sys.exit(0)
l = r.l
l.vla_octo_load.restype = ctypes.c_void_p
l.vla_octo_load.argtypes = [ctypes.c_char_p, ctypes.c_char_p]
l.vla_octo_predict.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int32, ctypes.c_void_p, ctypes.c_char_p,
                                                       ctypes.c_uint64, ctypes.c_int32, ctypes.c_void_p]
l.vla_octo_free.argtypes = [ctypes.c_void_p]
h = l.vla_octo_load(%(ckpt)r.encode(), (%(ckpt)r + "/tok").encode())
out = np.zeros((sh.horizon, sh.action_dim), np.float32)
P = lambda a: a.ctypes.data_as(ctypes.c_void_p)
def query(i):
    # a control loop's sliding window: one new frame per call (the reference
    # reuses the stem output of the frame it saw last call)
    p = np.ascontiguousarray(prim[i:i + sh.window]); w = np.ascontiguousarray(wrist[i:i + sh.window])
    return l.vla_octo_predict(h, P(p), P(w), sh.window, P(tm), ins.encode(), i, 1, P(out))
query(0)
times = []
t_end = time.perf_counter() + budget
while len(times) < max_steps and (not times or time.perf_counter() < t_end):
    t0 = time.perf_counter()
    rc = query(len(times) + 1)
    times.append(time.perf_counter() - t0)
    assert rc == 0
l.vla_octo_free(h)
print(json.dumps({"steps": len(times), "seconds": sum(times), "p50_ms": 1e3 * float(np.median(times))}))
"""


def time_reference_octo_cpu(ckpt: str, budget_s: float, max_steps: int):
    """The reference's own Octo query (oracle/_ref) in a fresh process, all host cores."""
    cores = cpu_cores()
    env = dict(os.environ, OCTO_INT8=str(OCTO_MASK), OMP_NUM_THREADS=str(cores), OMP_PROC_BIND="close",
               CUDA_VISIBLE_DEVICES="")
    code = _OCTO_CPU_CHILD % {"root": ROOT, "budget": budget_s, "max_steps": max_steps, "ckpt": ckpt}
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=900)
    if r.returncode != 0:
        return {"unavailable": f"reference CPU run failed: {r.stderr.strip().splitlines()[-1:]}"}
    d = json.loads(r.stdout.strip().splitlines()[-1])
    if "unavailable" in d:
        return d
    d["cores"] = cores
    d["chunks_per_s"] = d["steps"] / d["seconds"]
    return d


def run_octo(args):
    """Octo-base-shaped policy: one query batch per step (2-frame window of a
    256x256 primary and a 128x128 wrist camera, one instruction whose T5
    encoding is cached, DDPM 20); replicas per GPU."""
    import torch
    rank, local_rank, world = _env_rank()
    os.environ["VLA_CUDA_DEVICE"] = str(local_rank)
    os.environ["OCTO_INT8"] = str(OCTO_MASK)
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    from vla_simd_b200 import OctoPolicy, synth
    B = args.batch
    sh = synth.OCTO_BASELINE
    ckpt_root = tempfile.mkdtemp(prefix="vla_octo_")
    ckpt = synth.write_octo_checkpoint(os.path.join(ckpt_root, "octo"), sh, seed=0)
    pol = OctoPolicy(ckpt, max_batch=B)
    p, w, tm, ins, noise, z = synth.octo_inputs(sh, seed=1 + rank, batch=B)
    ins = [synth.octo_instruction(1)] * B
    pol.predict_batch(p, w, tm, ins, noise, z)   # leaves the batch resident in the device input buffers
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(device=dev)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    for _ in range(max(args.warmup, 3)):
        pol.enqueue(B, sh.window, True, stream.cuda_stream)
    torch.cuda.synchronize()
    kernels = pol.kernels_per_step
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        for i in range(args.steps):
            with torch.cuda.stream(stream):
                flush.zero_()
            starts[i].record(stream)
            pol.enqueue(B, sh.window, True, stream.cuda_stream)
            ends[i].record(stream)
        torch.cuda.synchronize()
    if dist:
        dist.barrier()
    step_s = [s_.elapsed_time(e_) * 1e-3 for s_, e_ in zip(starts, ends)]
    total_max = max_over_ranks(sum(step_s), dist, dev)
    value = job_value(args.steps * B, world, total_max)
    # end to end through the C ABI: host frames (a sliding window, a new frame
    # per call), noise and z in, host actions out
    n_e2e = max(args.steps, 10)
    rng = np.random.default_rng(11 + rank)
    seq_p = rng.integers(0, 256, size=(n_e2e + 3, B, 256, 256, 3), dtype=np.uint8)
    seq_w = rng.integers(0, 256, size=(n_e2e + 3, B, 128, 128, 3), dtype=np.uint8)

    def window(i):
        return (np.ascontiguousarray(seq_p[i:i + sh.window].transpose(1, 0, 2, 3, 4)),
                np.ascontiguousarray(seq_w[i:i + sh.window].transpose(1, 0, 2, 3, 4)))
    wins = [tuple(pinned(torch, a) for a in window(i)) for i in range(n_e2e + 2)]
    tm_h, noise_h, z_h = pinned(torch, tm), pinned(torch, noise), pinned(torch, z)
    for i in range(2):
        pol.predict_batch(wins[i][0], wins[i][1], tm_h, ins, noise_h, z_h)
    if dist:
        dist.barrier()
    calls = timed_calls(lambda i: pol.predict_batch(wins[i + 2][0], wins[i + 2][1], tm_h, ins, noise_h, z_h), n_e2e)
    e2e_s = max_over_ranks(sum(calls), dist, dev)
    e2e = {"value": job_value(n_e2e * B, world, e2e_s), "unit": "chunks/s",
           "h2d_bytes_per_step": p.nbytes + w.nbytes + tm.nbytes + noise.nbytes + z.nbytes + 4 * B,
           "d2h_bytes_per_step": B * sh.flat * 4, "p50_ms_per_call": 1e3 * statistics.median(calls),
           "path": "vla_octo_predict_batch (C ABI), pinned host frames + masks + noise -> host actions"}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:   # the CPU baseline runs at N=1 only
        cpu = time_reference_octo_cpu(ckpt, budget_s=args.cpu_budget, max_steps=20)
    pol.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    cpu_baseline = None
    if cpu and "unavailable" not in cpu:
        cpu_baseline = {"value": round(cpu["chunks_per_s"], 3), "unit": "chunks/s", "cores": cpu["cores"],
                        "kind": "reference", "p50_ms": round(cpu["p50_ms"], 2),
                        "sample": f"{cpu['steps']} single queries (same checkpoint, OCTO_INT8={OCTO_MASK}, a "
                                  f"sliding 2-frame window) of the reference's own vla_octo_predict, "
                                  f"OMP_NUM_THREADS={cpu['cores']}"}
    elif cpu:
        cpu_baseline = {"unavailable": cpu["unavailable"]}
    print(json.dumps({
        "metric": "Octo throughput (chunks/s)", "value": round(value, 3), "unit": "chunks/s",
        "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3),
        "ms_per_step": round(1e3 * total_max / args.steps, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8 (W8A8 GEMMs, int32 acc) + fp32",
        "data": "synthetic (seeded random-init Octo weights, uniform uint8 frames, N(0,1) noise, a synthetic "
                "T5 vocabulary)",
        "config": {"workload": "Octo-base-shaped: 12 layers d768 12 heads MLP 3072, 2-frame window of 256x256 "
                               "primary + 128x128 wrist (256 + 64 tokens per frame), T5-base text tower over 16 "
                               "tokens (cached per instruction), 20-step DDPM head, 4x7 chunk",
                   "batch_per_gpu": B, "int8_mask": OCTO_MASK, "parallelism": f"replicas x{world} (no collective)",
                   "l2": "flushed between steps (256 MiB memset outside the timed events)"},
        "latency_ms": {"p50": round(1e3 * statistics.median(step_s), 4),
                       "p95": round(1e3 * float(np.percentile(step_s, 95)), 4)},
        "cpu_baseline": cpu_baseline, "e2e": e2e, "gpu_launches": kernels * args.steps,
        "kernels_per_step": kernels, "clocks": clk.summary(),
    }), flush=True)


SMOLVLA_MASK = 63   # SMOLVLA_INT8: vision, text tower and action expert GEMMs in W8A8

_SMOLVLA_CPU_CHILD = r"""
import ctypes, json, os, sys, time
sys.path.insert(0, %(root)r)
import numpy as np
from vla_simd_b200 import synth
budget, max_steps = %(budget)f, %(max_steps)d
sh = synth.SMOLVLA_BASELINE
f, ins, st, nz = synth.smolvla_inputs(sh, seed=1)
from oracle import oracle
r = oracle.reference()
if r is None:
    print(json.dumps({"unavailable": "oracle/_ref/libvla_ref.so (the reference's own build) not present"}))
    sys.exit(0)
l = r._smolvla_bind()
h = l.vla_smolvla_load(%(ckpt)r.encode(), (%(ckpt)r + "/tok").encode())
n = l.vla_smolvla_tok_maxlen(h)
ids, mask = np.zeros(n, np.int32), np.zeros(n, np.int32)
l.vla_smolvla_tokenize(h, ins.encode(), ids.ctypes.data_as(ctypes.c_void_p), mask.ctypes.data_as(ctypes.c_void_p))
out = np.zeros((sh.chunk, sh.action_dim), np.float32)
P = lambda a: a.ctypes.data_as(ctypes.c_void_p)
def query():
    return l.vla_smolvla_predict_rtc(h, P(f), sh.n_views, sh.frame_h, sh.frame_w, P(ids), P(mask), n, P(st), P(nz),
                                     0, P(out), None, 0, None, 0.0)
query()
times = []
t_end = time.perf_counter() + budget
while len(times) < max_steps and (not times or time.perf_counter() < t_end):
    t0 = time.perf_counter()
    rc = query()
    times.append(time.perf_counter() - t0)
    assert rc == 0
l.vla_smolvla_free(h)
print(json.dumps({"steps": len(times), "seconds": sum(times), "p50_ms": 1e3 * float(np.median(times))}))
"""


def run_smolvla(args):
    """SmolVLA-shaped policy: one query batch per step (2 views of 480x640
    camera frames resized and padded to 512, a 48-token prompt, state, 10
    flow-matching steps); replicas per GPU. Device-timed value and C-ABI e2e."""
    import torch
    rank, local_rank, world = _env_rank()
    os.environ["VLA_CUDA_DEVICE"] = str(local_rank)
    os.environ["SMOLVLA_INT8"] = str(SMOLVLA_MASK)
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    from vla_simd_b200 import SmolvlaPolicy, synth
    B = args.batch
    sh = synth.SMOLVLA_BASELINE
    ckpt_root = tempfile.mkdtemp(prefix="vla_smolvla_")
    ckpt = synth.write_smolvla_checkpoint(os.path.join(ckpt_root, "smolvla"), sh, seed=0)
    pol = SmolvlaPolicy(ckpt, max_batch=B)
    f, ins, st, nz = synth.smolvla_inputs(sh, seed=1 + rank, batch=B)
    f, st, nz = pinned(torch, f), pinned(torch, st), pinned(torch, nz)
    for _ in range(max(args.warmup, 3)):
        pol.predict_batch(f, ins, st, nz)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    n = max(args.steps, 5)
    step_s = []
    with ClockSampler(local_rank) as clk:
        for _ in range(n):
            t0 = time.perf_counter()
            pol.predict_batch(f, ins, st, nz)
            step_s.append(time.perf_counter() - t0)
    total = max_over_ranks(sum(step_s), dist, dev)
    value = job_value(n * B, world, total)
    kernels = pol.kernels_per_step
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:   # the CPU baseline runs at N=1 only
        cpu = time_reference_generic(_SMOLVLA_CPU_CHILD, ckpt, "SMOLVLA_INT8", SMOLVLA_MASK, args.cpu_budget, 10)
    pol.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    cpu_baseline = None
    if cpu and "unavailable" not in cpu:
        cpu_baseline = {"value": round(cpu["chunks_per_s"], 3), "unit": "chunks/s", "cores": cpu["cores"],
                        "kind": "reference", "p50_ms": round(cpu["p50_ms"], 2),
                        "sample": f"{cpu['steps']} single queries (same checkpoint and inputs, SMOLVLA_INT8="
                                  f"{SMOLVLA_MASK}) of the reference's own vla_smolvla_predict_rtc, "
                                  f"OMP_NUM_THREADS={cpu['cores']}"}
    elif cpu:
        cpu_baseline = {"unavailable": cpu["unavailable"]}
    print(json.dumps({
        "metric": "SmolVLA throughput (chunks/s)", "value": round(value, 3), "unit": "chunks/s", "n_gpus": world,
        "steps": n, "warmup": max(args.warmup, 3), "ms_per_step": round(1e3 * total / n, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8 (W8A8 GEMMs, int32 acc) + fp32",
        "data": "synthetic (seeded random-init SmolVLA-shaped weights, uniform uint8 frames, N(0,1) state and noise, "
                "a synthetic BPE vocabulary)",
        "config": {"workload": "SmolVLA-shaped: SigLIP 12 layers d768 at 512 px -> 64 tokens per view x 2 views "
                               "(480x640 frames resized with pad), SmolLM2 16 layers h960 15/5 heads, 48 prompt "
                               "tokens + state, expert 16 layers h720, 10 flow-matching steps, 50 x 6 chunk",
                   "batch_per_gpu": B, "int8_mask": SMOLVLA_MASK,
                   "parallelism": f"replicas x{world} (no collective)",
                   "timing": "wall clock per vla_smolvla_predict_batch call (pinned host frames in, host actions "
                             "out: this line's value is already end to end)"},
        "latency_ms": {"p50": round(1e3 * statistics.median(step_s), 4)},
        "cpu_baseline": cpu_baseline,
        "e2e": {"value": round(value, 3), "unit": "chunks/s", "h2d_bytes_per_step": f.nbytes + st.nbytes + nz.nbytes,
                "d2h_bytes_per_step": B * sh.chunk * sh.action_dim * 4},
        "gpu_launches": kernels * n, "kernels_per_step": kernels, "clocks": clk.summary(),
    }), flush=True)


def time_reference_generic(child: str, ckpt: str, env_key: str, mask: int, budget_s: float, max_steps: int):
    """A reference policy's own query (oracle/_ref) timed in a fresh process on all host cores."""
    cores = cpu_cores()
    env = dict(os.environ, OMP_NUM_THREADS=str(cores), OMP_PROC_BIND="close", CUDA_VISIBLE_DEVICES="")
    env[env_key] = str(mask)
    code = child % {"root": ROOT, "budget": budget_s, "max_steps": max_steps, "ckpt": ckpt}
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=900)
    if r.returncode != 0:
        return {"unavailable": f"reference CPU run failed: {r.stderr.strip().splitlines()[-1:]}"}
    d = json.loads(r.stdout.strip().splitlines()[-1])
    if "unavailable" in d:
        return d
    d["cores"] = cores
    d["chunks_per_s"] = d["steps"] / d["seconds"]
    return d


def run_reference(args):
    """Reference arm: the reference's own CPU implementation on this host (rank 0 only)."""
    rank, _, world = _env_rank()
    if rank != 0:
        return
    from vla_simd_b200 import synth
    ckpt_root = tempfile.mkdtemp(prefix="vla_act_ref_")
    ckpt = synth.write_act_checkpoint(os.path.join(ckpt_root, "act"), synth.ACT_BASELINE, seed=0)
    steps = args.steps
    warmup = max(args.warmup, 3)
    cpu = time_reference_cpu(ckpt, budget_s=max(10.0, args.cpu_budget), max_steps=steps, warmup=warmup)
    if "unavailable" in cpu:
        print(json.dumps({"impl": "reference", "unavailable": cpu["unavailable"]}), flush=True)
        return
    v = cpu["chunks_per_s"]
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "chunks/s", "n_gpus": world,
        "steps": cpu["steps"], "warmup": warmup, "ms_per_step": round(1e3 * cpu["seconds"] / cpu["steps"], 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8 (W8A8) + fp32 (CPU)",
        "data": "synthetic (seeded random-init ACT weights)",
        "config": {"workload": "ACT policy step, BASELINE configs[1] (same checkpoint and inputs as ours)",
                   "int8_mask": INT8_MASK, "parallelism": "CPU, OpenMP over all host cores"},
        "cpu_baseline": {"value": round(v, 3), "unit": "chunks/s", "cores": cpu["cores"], "kind": "reference",
                         "sample": f"{cpu['steps']} steps of vla_act_predict from oracle/_ref", "cpu": cpu_model()},
        "e2e": {"value": round(v, 3), "unit": "chunks/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "latency_ms": {"p50": round(cpu["p50_ms"], 3)},
    }), flush=True)


def timeline_table(events, nsteps: int, top: int = 30):
    """Per-kernel marginal device time of the profiled steps: kernels in order
    of their end, each charged its end minus the latest earlier end (under
    programmatic dependent launch a kernel starts before its predecessor ends,
    so its own duration overstates what it adds to the step)."""
    import collections
    ks = sorted(events, key=lambda k: k[1])
    inc = collections.defaultdict(lambda: [0, 0.0])
    prev = ks[0][0]
    for s_, e_, name in ks:
        key = name.replace("(anonymous namespace)::", "").replace("vsb::", "").split("(")[0]
        key = key[5:] if key.startswith("void ") else key
        inc[key][0] += 1
        inc[key][1] += max(0.0, e_ - prev)
        prev = max(prev, e_)
    total = sum(v[1] for v in inc.values())
    rows = sorted(inc.items(), key=lambda x: -x[1][1])[:top]
    return total / nsteps, [(k, c / nsteps, t / nsteps, t / c, t / total) for k, (c, t) in rows]


def run_timeline(args):
    """One GPU: profile graph replays of the ACT step (or SmolVLA queries) with
    CUPTI (torch.profiler) and print each kernel's marginal time per step."""
    import torch
    from torch.profiler import profile, ProfilerActivity
    torch.cuda.set_device(0)
    n = max(args.steps, 1) if args.steps <= 20 else 5
    if args.model == "smolvla":
        os.environ["SMOLVLA_INT8"] = str(SMOLVLA_MASK)
        from vla_simd_b200 import SmolvlaPolicy, synth
        sh = synth.SMOLVLA_BASELINE
        pol = SmolvlaPolicy(synth.write_smolvla_checkpoint(os.path.join(tempfile.mkdtemp(), "s"), sh, seed=0),
                            max_batch=args.batch)
        f, ins, st_, nz = synth.smolvla_inputs(sh, seed=1, batch=args.batch)
        step = lambda: pol.predict_batch(f, ins, st_, nz)  # noqa: E731
    elif args.model == "dp":
        os.environ["DIFFUSION_INT8"] = str(DP_MASK)
        from vla_simd_b200 import DiffusionPolicy, synth
        pol = DiffusionPolicy(synth.write_dp_checkpoint(os.path.join(tempfile.mkdtemp(), "d"), synth.DP_BASELINE,
                                                        seed=0), max_batch=args.batch)
        frames, state, noise = synth.dp_inputs(synth.DP_BASELINE, seed=1, batch=args.batch)
        pol.predict_batch(frames, state, noise)
        stream = torch.cuda.Stream()
        step = lambda: pol.enqueue(args.batch, stream.cuda_stream)  # noqa: E731
    elif args.model == "octo":
        os.environ["OCTO_INT8"] = str(OCTO_MASK)
        from vla_simd_b200 import OctoPolicy, synth
        sh = synth.OCTO_BASELINE
        pol = OctoPolicy(synth.write_octo_checkpoint(os.path.join(tempfile.mkdtemp(), "o"), sh, seed=0),
                         max_batch=args.batch)
        p_, w_, tm, ins, noise, z = synth.octo_inputs(sh, seed=1, batch=args.batch)
        pol.predict_batch(p_, w_, tm, [synth.octo_instruction(1)] * args.batch, noise, z)
        stream = torch.cuda.Stream()
        step = lambda: pol.enqueue(args.batch, sh.window, True, stream.cuda_stream)  # noqa: E731
    else:
        os.environ["ACT_INT8"] = str(INT8_MASK)
        from vla_simd_b200 import ActPolicy, synth
        pol = ActPolicy(synth.write_act_checkpoint(os.path.join(tempfile.mkdtemp(), "a"), synth.ACT_BASELINE, seed=0))
        f, s_ = synth.act_inputs(synth.ACT_BASELINE, seed=1)
        pol.predict(f, s_)
        stream = torch.cuda.Stream()
        step = lambda: pol.enqueue(stream.cuda_stream)  # noqa: E731
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(n):
            step()
        torch.cuda.synchronize()
    ev = [(e.time_range.start, e.time_range.end, e.name) for e in prof.events()
          if e.device_type == torch.autograd.DeviceType.CUDA
          and not any(w in e.name.lower() for w in ("memset", "memcpy"))]
    per_step, rows = timeline_table(ev, n)
    print(f"# {args.model} step timeline: {len(ev) / n:.0f} kernels per step, {per_step:.1f} us per step "
          f"(marginal sum over {n} profiled steps, L2 warm)")
    print("| kernel | launches / step | us / step | us / launch | share |\n|---|---:|---:|---:|---:|")
    for k, c, t, tl, fr in rows:
        print(f"| `{k}` | {c:.1f} | {t:.1f} | {tl:.2f} | {100 * fr:.1f}% |")
    pol.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-budget", type=float, default=15.0, help="seconds of reference CPU steps")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--op", default=None, help="time one op at its ACT shape (attention, gemm_qkv, gemm_w1, "
                                               "gemm_w2, layernorm, quantize, conv_layer1), or gemm_msweep "
                                               "(the FFN GEMM at M = 602 x {1, 8, 32, 128})")
    ap.add_argument("--model", choices=["act", "dp", "octo", "smolvla"], default="act",
                    help="act: the ACT step (the headline line); dp: Diffusion Policy (BASELINE configs[2]); "
                         "octo: the Octo-base-shaped policy; smolvla: the SmolVLA-shaped policy")
    ap.add_argument("--batch", type=int, default=1, help="queries per step per GPU (--model dp / octo)")
    ap.add_argument("--gemm-only", action="store_true",
                    help="time only the W8A8 GEMM at the ACT FFN shape (a small case for ncu captures)")
    ap.add_argument("--timeline", action="store_true",
                    help="profile a few steps (any --model, --batch) and print each kernel's marginal time")
    args = ap.parse_args()
    if args.timeline:
        run_timeline(args)
        return
    if args.op:
        run_op(args.op)
        return
    if args.gemm_only:
        import torch
        torch.cuda.set_device(0)
        print(json.dumps({"int8_gemm": time_gemm(torch, torch.device("cuda", 0), n_cold=5, n_warm_graph=5,
                                                 n_lin=2)}), flush=True)
        return
    if args.model == "dp" and args.impl != "reference":
        run_dp(args)
    elif args.model == "octo" and args.impl != "reference":
        run_octo(args)
    elif args.model == "smolvla" and args.impl != "reference":
        run_smolvla(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
