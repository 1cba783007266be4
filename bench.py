#!/usr/bin/env python
"""Benchmark of the BF16 projection hot path on B200: one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

A step is one projection y = x . W^T of the workload's shape. Default workload: the small-batch
QKV projection, x[16, 4096] . W[6144, 4096]^T (the configuration the metric is quoted on). Each
step uses the next of R distinct weight/input copies, R chosen so the copies exceed the 126 MB L2:
every step reads its weights cold from HBM, as the reference's judge does with its L2 flush.

`value` is whole-job throughput (algorithmic bytes / s for M <= 32, FLOP/s for M >= 128, as
reference.py:102-107 counts them) with inputs resident in HBM, timed with CUDA events on the
launching stream (max over ranks). `e2e` is the same metric through the public kernel_fn with the
inputs copied from pinned host memory and the output copied back every step. `roofline` is the
projection kernel's achieved rate per launch against MEASURED_PEAKS.json. `cpu_baseline` times
the reference's CPU path (its FP64 product, restated in numpy in oracle/contract_ref.py) on this
host on a bounded sample.

Multi-GPU (torchrun): the projection workloads run one independent replica per GPU ("weak"); the
mlp_up workloads shard W along N (column-parallel) so the total work is fixed ("strong").
`--impl reference` times the reference's CPU implementation (the FP64 numpy restatement, all
host threads) on the same workload; under torchrun only rank 0 runs it.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "proj latency µs + HBM TB/s (M≤32) / TFLOP/s (M≥128) at 1/2/4/8 B200"
L2_BYTES = 126 * 1024 * 1024
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}

WORKLOADS = {
    # name: (layer, M, weight recipe, weight format, sharded along N)
    "smallbatch_qkv": ("qkv_decode", 16, "normal", "bf16", False),
    "decode_qkv_gemv": ("qkv_decode", 1, "normal", "bf16", False),
    "gemv12_qkv": ("qkv_prefill", 1, "inject", "12b", False),
    "prefill_qkv": ("qkv_prefill", 4096, "normal", "bf16", False),
    "mlp_up_prefill": ("mlp_up", 8192, "normal", "bf16", True),
    "mlp_up_decode": ("mlp_up", 1, "normal", "bf16", True),
}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="smallbatch_qkv", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--m", type=int, default=0, help="override M (small-batch sweep)")
    ap.add_argument("--gather", default="", choices=["", "nccl", "fused"],
                    help="sharded workloads: also all-gather y, by NCCL after the projection or fused into its "
                         "epilogue (stores into every rank's y over NVLink)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--plan", default="", help="JSON plan overriding the dispatch table for this workload")
    return ap.parse_args()


def work_units(m: int, n: int, k: int, fmt: str, n_esc: int = 0) -> tuple[float, float]:
    """(algorithmic bytes, FLOPs) of one projection (reference.py:102-107; 12-bit: plane bytes,
    escape entries, row pointers and tile bases instead of 2 bytes a weight)."""
    if fmt == "12b":
        wbytes = n * k * 1.5 + 4 * n_esc + 4 * (n + 1) + math.ceil(n / 128) * (k // 128)
    else:
        wbytes = n * k * 2
    return wbytes + m * k * 2 + m * n * 2, 2.0 * m * n * k


def load_peaks() -> tuple[dict, str]:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def traffic_from_profiles(kernel: str, workload: str):
    """dram bytes per launch from the committed ncu summary profiles/<kernel>_<workload>.txt."""
    path = os.path.join(ROOT, "profiles", f"{kernel}_{workload}.txt")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        for line in f:
            if line.startswith("dram_bytes_per_launch:"):
                try:
                    return int(float(line.split(":", 1)[1].split()[0]))
                except ValueError:
                    return None
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 100 ms while running."""

    FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str | None):
        self.uuid = uuid
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100"]
            if self.uuid:
                cmd += ["-i", self.uuid]
            self.proc = subprocess.Popen(cmd, stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, ValueError):
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 10:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        mx = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[6 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def cpu_threads() -> int:
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
        return max(n) if n else os.cpu_count() or 1
    except Exception:  # noqa: BLE001 - only a label
        return os.cpu_count() or 1


class CpuReference:
    """The reference's CPU product (its FP64 ref_kernel, restated in numpy in oracle/contract_ref.py,
    the W to FP64 conversion included as reference.py:75 does it) on a bounded sample of the
    workload: all M rows of x, or 512 rows for prefill shapes."""

    def __init__(self, m, n, k):
        import numpy as np
        import torch

        from muse_bf16_proj_b200 import contract as C
        from oracle import contract_ref as O

        self.O = O
        self.rows = min(m, 512)
        g = torch.Generator().manual_seed(7)
        self.x = torch.randn((self.rows, k), generator=g).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
        self.w = (torch.randn((n, k), generator=g) * C.BASELINE_STD).to(torch.bfloat16).view(torch.int16).numpy().view(
            np.uint16)
        self.n, self.k = n, k
        O.ref_kernel(self.x[:1], self.w[: min(n, 256)])  # wake the BLAS threads

    def call(self) -> float:
        t0 = time.perf_counter()
        self.O.ref_kernel(self.x, self.w)
        return time.perf_counter() - t0

    def timed(self, seconds: float, max_calls: int, min_calls: int = 1) -> tuple[float, int]:
        times = []
        t_end = time.perf_counter() + seconds
        while len(times) < max_calls and (len(times) < min_calls or time.perf_counter() < t_end):
            times.append(self.call())
        return statistics.median(times), len(times)

    def sample(self, calls: int, sec: float) -> str:
        return (f"{calls} calls of the FP64 numpy product on x[{self.rows}, {self.k}] . W[{self.n}, {self.k}]^T "
                f"(W cast to FP64 each call, as reference.py:75), median {sec * 1e3:.1f} ms")


def main():
    args = parse_args()
    layer, m_default, recipe, fmt, sharded = WORKLOADS[args.workload]
    m = args.m or m_default
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    from muse_bf16_proj_b200 import contract as C
    n_full, k = C.BASELINE_LAYERS[layer]
    hbm_bound = m <= 32
    unit = "TB/s" if hbm_bound else "TFLOP/s"

    if args.impl == "reference":
        run_reference_arm(args, layer, m, recipe, fmt, sharded, n_full, k, rank, world, unit, hbm_bound)
        return

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    from muse_bf16_proj_b200 import _lib, submission
    from muse_bf16_proj_b200.dispatch import Dispatch

    # ---- workload: R rotating copies (each rank: its shard when sharded) ----------------------
    if sharded:
        from muse_bf16_proj_b200.sharded import shard_rows
        r0, r1 = shard_rows(n_full, world, rank)
        n = r1 - r0
    else:
        n, r0 = n_full, 0
    w_bytes = n * k * (1.5 if fmt == "12b" else 2)
    copy_bytes = w_bytes + m * k * 2 + m * n * 2
    rot = max(2, min(16, math.ceil(3 * L2_BYTES / copy_bytes)))
    if copy_bytes * rot > 40e9:
        rot = 2
    weights = {}
    for i in range(rot):
        w = C.generate_baseline_weight(layer, 1000 + i, device=str(dev), recipe=recipe)
        weights[f"{layer}_{i}"] = w[r0:r0 + n].contiguous() if sharded else w
        del w
    torch.cuda.empty_cache()
    entries = None
    if fmt == "12b" and not Dispatch().wants_12b(n, k):  # no table row: the library's 12-bit tile plan
        entries = [{"n": n, "k": k, "m_lo": m, "m_hi": m, "weights": "12b",
                    "plan": _lib.plan_default(m, n, k, weights_12b=True, tiles=True).as_dict()}]
    if args.plan:
        entries = [{"n": n, "k": k, "m_lo": m, "m_hi": m, "weights": fmt, "plan": json.loads(args.plan)}]
    disp = Dispatch(entries=entries) if entries is not None else Dispatch()
    state = submission.prepare(weights, dispatch=disp, encode_12b=(fmt == "12b"), verbose=False)
    names = list(weights)
    xs = [C.generate_input(m, layer, 2000 + i, device=str(dev))["x"] for i in range(rot)]
    ys = [torch.empty((m, n), dtype=torch.bfloat16, device=dev) for _ in range(rot)]
    n_esc = state["enc12"][names[0]].n_esc if fmt == "12b" else 0
    plan, plan_fmt = state["dispatch"].plan(m, n, k, fmt == "12b")
    assert plan_fmt == fmt, (plan_fmt, fmt)
    bytes_step, flops_step = work_units(m, n, k, fmt, n_esc)
    stream = torch.cuda.current_stream(dev)

    def step(i):
        j = i % rot
        submission.project(xs[j], state, names[j], n, out=ys[j])

    gather_out = None
    if sharded and args.gather == "nccl" and world > 1:
        from muse_bf16_proj_b200.sharded import gather_columns
        gather_out = torch.empty((m, n_full), dtype=torch.bfloat16, device=dev)
    fused = None
    if sharded and args.gather == "fused":
        from muse_bf16_proj_b200.sharded import FusedGatherProjection
        fused = FusedGatherProjection(weights[names[0]], n_full, max_rows=m, shard_given=True)
        plan = fused.plan(m)
        if any(name not in state["tiles"] for name in names):
            raise RuntimeError("the fused all-gather needs the packed tiles of every rotating weight")

        def step(i):  # noqa: F811 - the projection with the all-gather in its epilogue
            j = i % rot
            fused.project(xs[j], plan=plan, tiles=state["tiles"][names[j]])

    # ---- warm-up, clock soak, timed region --------------------------------------------------
    for i in range(max(3, args.warmup)):
        step(i)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(rot):
        step(i)
    torch.cuda.synchronize()
    enqueue_s = (time.perf_counter() - t0) / rot  # host cost of one step (upper bound)
    props = torch.cuda.get_device_properties(dev)
    sampler = ClockSampler("GPU-" + str(props.uuid) if getattr(props, "uuid", None) else None)
    sampler.start()
    soak_end = time.perf_counter() + 1.5
    i = 0
    if world > 1:
        # Every rank makes the same number of calls (the fused all-gather pairs each rank's call
        # with its peers'): the soak's length is agreed as a step count, not a deadline.
        n_soak = torch.tensor([max(32, min(20000, int(1.5 / max(enqueue_s, 1e-6))))], device=dev)
        dist.all_reduce(n_soak, op=dist.ReduceOp.MIN)
        for i in range(int(n_soak[0])):
            step(i)
            if i % 32 == 31:
                torch.cuda.synchronize()
        torch.cuda.synchronize()
    while world == 1 and time.perf_counter() < soak_end:
        for _ in range(32):
            step(i)
            i += 1
        torch.cuda.synchronize()

    K = args.steps
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    # Keep the GPU busy while the host enqueues every step, so the timed region holds no host gaps.
    # Only the region's two events: an event between steps would stop the next projection's
    # programmatic launch from overlapping the previous one, as it does in a serving stream.
    torch.cuda._sleep(int(min(2e9, (K * (enqueue_s + 20e-6) + 2e-3) * 2.0e9)))
    torch.cuda.nvtx.range_push("bench_timed")  # lets `ncu --nvtx --nvtx-include bench_timed/` list these launches
    start.record(stream)
    for i in range(K):
        step(i)
        if gather_out is not None:
            gather_columns(ys[i % rot], world, out=gather_out)
    end.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    total_ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([total_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t[0])
    # One projection kernel per step: its launch-to-launch time is the step time.
    mean_launch_ms = total_ms / K
    isolated_us = isolated_latency_us(step, rot, stream)
    code = _lib.device_error(stream.cuda_stream)

    # ---- e2e through kernel_fn with host buffers --------------------------------------------
    e2e = run_e2e(state, names, layer, m, n, k, rot, K, dev, world, bytes_step, flops_step)
    accuracy = measure_accuracy(state, names[0], weights[names[0]], xs[0], n)

    if fused is not None:
        fused.close()  # every rank: unmap the peers' buffers before any rank frees its own
    if world > 1:
        dist.barrier()
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return

    per_step_ms = total_ms / K
    # Every rank runs K projections of its own shape (a replica, or its N/world shard): the job
    # moves world x the per-rank bytes (FLOPs) in the slowest rank's time.
    value = world * (bytes_step if hbm_bound else flops_step) * K / (total_ms * 1e-3) / 1e12
    peaks, peaks_kind = load_peaks()
    kernel_name = _lib.KERNEL_NAMES.get(plan.kernel, str(plan.kernel))
    if hbm_bound:
        achieved = bytes_step / (mean_launch_ms * 1e-3) / 1e9
        peak = peaks["hbm_gbs"]
        roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "algorithmic_bytes_per_launch": int(bytes_step)}
    else:
        # Back-to-back steps keep the GPU under sustained load (power cap): the sustained GEMM
        # figure is the denominator; the isolated single launch is held against the burst one.
        achieved = flops_step / (mean_launch_ms * 1e-3) / 1e12
        peak = peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
        burst = flops_step / (isolated_us * 1e-6) / 1e12
        roof = {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                "frac": round(achieved / peak, 4), "algorithmic_flops_per_launch": flops_step,
                "peak_kind": "sustained (bf16_tflops_sustained)",
                "isolated_achieved": round(burst, 1), "isolated_frac_of_burst": round(burst / peaks["bf16_tflops"], 4)}
    roof["peak_source"] = f"{peaks_kind} (MEASURED_PEAKS.json)" if peaks_kind == "measured" else "fallback"
    roof["kernel"] = kernel_name
    roof["mean_launch_us"] = round(mean_launch_ms * 1e3, 3)
    roof["launch_time"] = "timed region / steps (one projection kernel per step, launched back to back)"
    roof["traffic"] = traffic_from_profiles(kernel_name, args.workload)
    roof["spec_frac"] = round(achieved / (8000.0 if hbm_bound else 2250.0), 4)

    line = {
        "metric": METRIC, "value": round(value, 4), "unit": unit, "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": round(per_step_ms, 6), "latency_us": round(per_step_ms * 1e3, 3),
        "isolated_launch_us": round(isolated_us, 3),
        "higher_is_better": True, "scaling": "strong" if sharded else "weak", "vs_baseline": None,
        "dtype": "bf16" if fmt == "bf16" else "bf16 (12-bit lossless weights)",
        "data": "synthetic: seeded x ~ N(0,1) with the reference's probe rows, W ~ N(0,0.02)"
                + (" with 0.1% injected zeros/x50 outliers" if recipe == "inject" else ""),
        "config": {"workload": args.workload, "m": m, "n": n_full, "k": k, "n_per_gpu": n,
                   "weights": fmt, "plan": plan.as_dict(),
                   "l2": f"{rot} rotating weight/input copies ({rot * copy_bytes / 1e6:.0f} MB) > 126 MB L2",
                   "parallelism": (f"column-parallel N/{world}" if sharded else f"replicas x{world}")},
        "roofline": roof,
        "e2e": e2e,
        "gpu_launches": K,
        "clocks": clocks,
        "device_error": code,
        "accuracy": accuracy,
    }
    if gather_out is not None:
        line["config"]["all_gather"] = ("NCCL all_gather_into_tensor of y into [P, M, N/P] plus the copy to [M, N] "
                                        "after every step, inside the timed region")
    if fused is not None:
        line["config"]["all_gather"] = ("fused into the projection's epilogue: every output value stored into all "
                                        f"{world} ranks' y [M, N] over NVLink (CUDA IPC peers), flag barrier per call")
        # The slower of the GEMM and the link: this rank's slice to each of the other ranks.
        link_bytes = (world - 1) * m * n * 2
        link_peak = 770.0  # GB/s per direction per GPU, measured peer copy on this pool's B200s
        t_link = link_bytes / (link_peak * 1e9)
        t_math = (bytes_step / (peaks["hbm_gbs"] * 1e9)) if hbm_bound else flops_step / (peak * 1e12)
        line["roofline"]["fused_gather"] = {
            "nvlink_bytes_per_rank_per_step": link_bytes, "link_peak_gbs": link_peak,
            "link_achieved_gbs": round(link_bytes / (mean_launch_ms * 1e-3) / 1e9, 1),
            "target_us": round(max(t_link, t_math) * 1e6, 3),
            "frac_of_target": round(max(t_link, t_math) / (mean_launch_ms * 1e-3), 4)}
    if world == 1 and not args.no_cpu_baseline:
        cpu = CpuReference(m, n, k)
        sec, calls = cpu.timed(args.cpu_seconds, max_calls=30)
        b, f = work_units(cpu.rows, n, k, "bf16")
        line["cpu_baseline"] = {"value": (b if hbm_bound else f) / sec / 1e12, "unit": unit, "cores": cpu_threads(),
                                "kind": "port", "sample": cpu.sample(calls, sec)}
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def isolated_latency_us(step, rot, stream, reps: int = 20) -> float:
    """Median time of ONE projection launch with nothing queued around it and its weights cold
    in L2 (the next copy of the rotation), as the reference's judge times a call (its ~4 us graph
    replay cost is not subtracted here)."""
    import torch

    times = []
    for i in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        torch.cuda._sleep(200000)  # ~0.1 ms: the launch is enqueued before the first event fires
        a.record(stream)
        step(i)
        b.record(stream)
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b) * 1e3)
    return statistics.median(times)


def measure_accuracy(state, name, w, x, n) -> dict:
    """Max-abs and relative-L2 error of one projection (this rank's shard) against a torch FP64
    product of the same x and W on the GPU, as the reference computes its expected output
    (reference.py:72-76, before the BF16 rounding), and the largest difference from that product
    rounded to BF16. Runs after the timed region."""
    import torch

    from muse_bf16_proj_b200 import submission

    y = submission.project(x, state, name, n).double()
    ref = x.double() @ w[:n].double().t()
    err = y - ref
    return {"max_abs": float(err.abs().max()), "rel_l2": float(err.norm() / ref.norm().clamp(min=1e-300)),
            "max_abs_vs_bf16_rounded_ref": float((y - ref.to(torch.bfloat16).double()).abs().max()),
            "ref": "torch FP64 x . W^T on the GPU (reference.py:72-76); one step, this rank's shard"}


def run_e2e(state, names, layer, m, n, k, rot, K, dev, world, bytes_step, flops_step):
    """The same projections through the public kernel_fn with host buffers: each step copies x in
    from pinned host memory, calls kernel_fn and copies y back to pinned host memory. The three
    are captured once per weight copy into a CUDA graph and replayed, as the reference's harness
    runs kernel_fn (validate.py:124-147); `eager_us_per_step` is the same loop without graphs."""
    import torch

    from muse_bf16_proj_b200 import contract as C
    from muse_bf16_proj_b200 import submission

    hx = [C.generate_input(m, layer, 3000 + i, device="cpu")["x"].pin_memory() for i in range(rot)]
    hy = [torch.empty((m, n), dtype=torch.bfloat16).pin_memory() for _ in range(rot)]
    dx = [torch.empty((m, k), dtype=torch.bfloat16, device=dev) for _ in range(rot)]

    def one(j):
        dx[j].copy_(hx[j], non_blocking=True)
        y = submission.kernel_fn({"x": dx[j], "config": {"m": m, "n": n, "k": k, "layer": names[j]}}, state)
        hy[j].copy_(y, non_blocking=True)

    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for j in range(rot):
            one(j)
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize()
    graphs = []
    for j in range(rot):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            one(j)
        graphs.append(g)
    stream = torch.cuda.current_stream(dev)
    steps = max(K, 10)

    def timed(fn):
        for i in range(3):
            fn(i)
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        start.record(stream)
        for i in range(steps):
            fn(i)
        end.record(stream)
        torch.cuda.synchronize()
        return start.elapsed_time(end) / steps, (time.perf_counter() - t0) / steps

    per_ms, wall = timed(lambda i: graphs[i % rot].replay())
    eager_ms, _ = timed(lambda i: one(i % rot))
    del graphs

    # Serving loop: the same per-step work (x in, kernel_fn, y out), pipelined in groups of
    # `group` steps. A group's x copies run on a side stream while the previous group projects;
    # its projections then run back to back on the capturing stream (kernel_fn allocates y
    # there), joined to the copies once a group rather than once a step, so consecutive
    # projections keep their programmatic-launch overlap; its y copies run on a second side stream
    # while the next group projects. Device x buffers form a ring of `depth` groups: a group's copies
    # wait for the projections that read its buffers `depth` groups before. A graph holds `chain`
    # steps; the longest chain whose outputs fit in 4 GiB, at least 32. Where a step's copies
    # outweigh its projection (MBs a step: prefill), a join costs nothing beside them but a group's
    # copies drain at the end of every graph, so those steps go one to a group with a ring of four.
    y_bytes = m * n * 2
    group, depth = (8, 2) if (m * k * 2 + y_bytes) <= (16 << 20) else (1, 4)
    chain = max(32, -(-rot // group) * group)
    while chain < 128 and 2 * chain * y_bytes <= (4 << 30):
        chain *= 2
    ring = [torch.empty((m, k), dtype=torch.bfloat16, device=dev) for _ in range(depth * group)]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    keep = []

    def pipeline():
        cap = torch.cuda.current_stream(dev)
        s_in.wait_stream(cap)
        s_out.wait_stream(cap)
        done = []  # per group: its last projection has run
        for g0 in range(0, chain, group):
            gi = g0 // group
            with torch.cuda.stream(s_in):
                if gi >= depth:
                    s_in.wait_event(done[gi - depth])
                for t in range(group):
                    ring[(gi % depth) * group + t].copy_(hx[(g0 + t) % rot], non_blocking=True)
                ev_in = torch.cuda.Event()
                ev_in.record(s_in)
            cap.wait_event(ev_in)
            ys = []
            for t in range(group):
                i = g0 + t
                y = submission.kernel_fn({"x": ring[(gi % depth) * group + t],
                                          "config": {"m": m, "n": n, "k": k, "layer": names[i % rot]}}, state)
                ys.append((i % rot, y))
            keep.extend(y for _, y in ys)
            ev = torch.cuda.Event()
            ev.record(cap)
            done.append(ev)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev)
                for j, y in ys:
                    hy[j].copy_(y, non_blocking=True)
        cap.wait_stream(s_in)
        cap.wait_stream(s_out)

    pg = torch.cuda.CUDAGraph()
    with torch.cuda.graph(pg):
        pipeline()
    reps = max(2, steps // chain)
    for _ in range(2):
        pg.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(reps):
        pg.replay()
    end.record(stream)
    torch.cuda.synchronize()
    pipe_ms = start.elapsed_time(end) / (reps * chain)
    del pg, keep
    # The host outputs of the last replay against one direct call per step slot: the pipelined
    # loop computed what kernel_fn computes.
    pipe_ok = True
    for j in range(rot):
        dx[j].copy_(hx[j])
        y = submission.kernel_fn({"x": dx[j], "config": {"m": m, "n": n, "k": k, "layer": names[j]}}, state)
        pipe_ok = pipe_ok and bool(torch.equal(y.cpu(), hy[j]))
    if world > 1:  # every rank takes the collective, then all raise together on any mismatch
        import torch.distributed as dist
        t = torch.tensor([per_ms, eager_ms, pipe_ms, 0.0 if pipe_ok else 1.0], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        per_ms, eager_ms, pipe_ms, pipe_ok = float(t[0]), float(t[1]), float(t[2]), float(t[3]) == 0.0
    if not pipe_ok:
        raise RuntimeError("pipelined serving loop: host outputs differ from direct kernel_fn calls")
    hbm = m <= 32
    val = world * (bytes_step if hbm else flops_step) / (pipe_ms * 1e-3) / 1e12
    return {"value": round(val, 4), "unit": "TB/s" if hbm else "TFLOP/s", "us_per_step": round(pipe_ms * 1e3, 3),
            "how": (f"serving loop through kernel_fn with host buffers: every step copies its x in from pinned host "
                    f"memory and its y out to pinned host memory; the copies run on two side streams in groups of "
                    f"{group} step{'s' if group > 1 else ''}, the next group's copies in and the previous group's copies out overlapping this "
                    f"group's back-to-back projections (graphs of {chain} steps; outputs checked against direct "
                    f"calls)"),
            "latency_us": round(per_ms * 1e3, 3),
            "latency_how": "one step alone, serial: graph replay of x in, kernel_fn, y out",
            "wall_us_per_step": round(wall * 1e6, 3), "eager_us_per_step": round(eager_ms * 1e3, 3),
            "h2d_bytes_per_step": m * k * 2, "d2h_bytes_per_step": m * n * 2}


def run_reference_arm(args, layer, m, recipe, fmt, sharded, n_full, k, rank, world, unit, hbm_bound):
    """The reference's own CPU path for this workload (FP64 numpy restatement, all host threads):
    W warm-up calls, then K timed calls (fewer if K would take over ~2 minutes)."""
    if rank != 0:
        return
    n = n_full // world if sharded else n_full
    cpu = CpuReference(m, n, k)
    first = cpu.call()
    steps = max(1, min(args.steps, int(120.0 / max(first, 1e-6))))
    for _ in range(args.warmup):
        cpu.call()
    times = [cpu.call() for _ in range(steps)]
    sec = statistics.median(times)
    b, f = work_units(cpu.rows, n, k, "bf16")
    value = (b if hbm_bound else f) / sec / 1e12
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": unit, "n_gpus": world,
            "steps": steps, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
            "scaling": "strong" if sharded else "weak", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic, same shapes and recipe", "config": {"workload": args.workload, "m": m, "n": n_full, "k": k},
            "cpu_baseline": {"value": value, "unit": unit, "cores": cpu_threads(), "kind": "port",
                             "sample": cpu.sample(steps, sec)},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
