"""Per-shape plan sweep on a B200: times every candidate plan and writes the dispatch table.

    python -m muse_bf16_proj_b200.sweep [--shapes reference,baseline] [--ms 1,2,...] [--out path]
                                        [--write-table] [--reps 40] [--flags 2] [--kernels a,b]
                                        [--plan JSON] [--trace] [--one-call REPS]

Replaces the reference's Optuna / grid sweeps (sweep_all.py, sweep_cuda.py) with a plain grid: for
each (N, K, M) every candidate plan is first checked against a torch FP32 product rounded to BF16
(TF32 off; relative L2 <= 1e-3), then timed over `reps` launches with CUDA events, each launch on the next
of R weight copies whose total exceeds the 126 MB L2 (every launch reads W cold from HBM, as the
reference's judge flushes L2). The fastest checked plan per shape becomes a table row; 12-bit
candidates are timed too and win a row only when faster than every BF16 plan. Every row also
records cuBLAS (torch F.linear) timed the same way on the same weights: the reference's scoring
baseline, kept as a comparator (never served). --one-call also times each candidate as the reference's
judge times a call (graph replay after an L2 flush); --trace records per-CTA timestamps and kernel marks.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import time

import numpy as np
import torch

from . import _lib, codec12
from .contract import BASELINE_LAYERS, LAYERS, UNPOOL_SLICE
from .dispatch import TABLE_PATH

L2_BYTES = 126 * 1024 * 1024

REFERENCE_SHAPES = [(LAYERS[n][0], LAYERS[n][1]) for n in ("qkv_gate", "o", "pooler", "unpooler")] + [(UNPOOL_SLICE, 4096)]
BASELINE_SHAPES = [BASELINE_LAYERS[n] for n in ("qkv_decode", "qkv_prefill")]
# The column-parallel MLP-up weight's per-GPU shards at 1, 2, 4 and 8 GPUs.
MLP_SHARD_SHAPES = [(BASELINE_LAYERS["mlp_up"][0] // p, BASELINE_LAYERS["mlp_up"][1]) for p in (1, 2, 4, 8)]
DEFAULT_MS = [1, 2, 4, 8, 16, 32, 64, 128, 256, 512]


def candidates(m: int, n: int, k: int, sms: int, twelve_ok: bool) -> list[tuple[str, _lib.MusePlan]]:
    """The plans worth timing at this shape: CUDA-core GEMVs at few tokens, the tile kernel with
    cluster or global split-K, and the stream-K kernel."""
    out = []
    if m <= 4 and k % 256 == 0:
        for warps, ctas in ((16, sms), (16, 2 * sms), (8, 2 * sms)):
            out.append(("bf16", _lib.MusePlan(kernel=_lib.KERNEL_GEMV_BF16, warps=warps, ctas=ctas, chunk=16)))
    if m <= 4:  # the register-streaming GEMV over the packed tiles (split 0: about 16 k blocks a warp)
        nkb = (k + 63) // 64
        for qw in (1, 2, 4, 8):
            for warps, split in ((8, 0), (4, 0), (16, 0), (8, 1), (16, 2), (16, 4), (8, 4), (4, 4), (16, 8)):
                if split <= nkb and (qw < 8 or m <= 2) and (qw > 1 or warps != 16 or split != 8):
                    out.append(("bf16", _lib.MusePlan(kernel=_lib.KERNEL_GEMV_TILES, warps=warps, split=split,
                                                      chunk=qw)))
    if twelve_ok and m <= 4:
        for warps, ctas in ((8, 2 * sms), (16, sms), (16, 2 * sms)):
            out.append(("12b", _lib.MusePlan(kernel=_lib.KERNEL_GEMV_12B, warps=warps, ctas=ctas)))
    b16 = 16
    while b16 < m and b16 < 128:
        b16 *= 2
    if twelve_ok and k % 512 == 0 and m <= 4:
        for per_sm in (0, 3, 4, 5, 6):
            for stages in (3, 4):
                out.append(("12b", _lib.MusePlan(kernel=_lib.KERNEL_GEMV_12T, ctas=per_sm * sms, stages=stages)))
    if twelve_ok and k % 512 == 0 and m <= 256:
        for stages in (0, 3):  # multiples of the decoder groups
            out.append(("12b", _lib.MusePlan(kernel=_lib.KERNEL_TC_12B, tile_n=b16, ctas=sms, stages=stages)))
    if m <= 256:
        for stages in (0, 4, 6):
            out.append(("bf16", _lib.MusePlan(kernel=_lib.KERNEL_TC_SKINNY, tile_n=b16, ctas=sms, stages=stages)))
    bnt = 16
    while bnt < m and bnt < 256:
        bnt *= 2
    nkb = (k + 63) // 64
    tiles = ((n + 127) // 128) * ((m + bnt - 1) // bnt)
    for split in (1, 2, 3, 4, 6, 8, 12, 16):
        if split > nkb or (split > 1 and tiles * split > 2 * sms) or (split == 1 and tiles < sms // 2 and nkb > 8):
            continue
        if split == 1:
            out.append(("bf16", _lib.MusePlan(kernel=_lib.KERNEL_TC_TILE, tile_n=bnt, split=1)))
            continue
        out.append(("bf16", _lib.MusePlan(kernel=_lib.KERNEL_TC_TILE, tile_n=bnt, split=split,
                                          flags=_lib.FLAG_GLOBAL_SPLIT)))
        if bnt <= 64:  # rings small enough for two CTAs an SM (the next launch's CTAs co-reside)
            for stages in (4, 6):
                out.append(("bf16", _lib.MusePlan(kernel=_lib.KERNEL_TC_TILE, tile_n=bnt, split=split, stages=stages,
                                                  flags=_lib.FLAG_GLOBAL_SPLIT)))
        if tiles * split <= sms:  # a cluster of `split` CTAs summing through DSMEM (all in one wave)
            out.append(("bf16", _lib.MusePlan(kernel=_lib.KERNEL_TC_TILE, tile_n=bnt, split=split)))
    if m >= 128:
        out.append(("bf16", _lib.MusePlan(kernel=_lib.KERNEL_TC_GEMM)))
        for group in (0, 16):  # token tiles walked together (0: as many as keep 32 MB of x)
            out.append(("bf16", _lib.MusePlan(kernel=_lib.KERNEL_TC_GEMM2, split=group)))
        if m <= 2048:  # few 256 x 256 tiles: the stream-K schedule keeps every CTA pair busy
            out.append(("bf16", _lib.MusePlan(kernel=_lib.KERNEL_TC_GEMM2, flags=_lib.FLAG_STREAMK)))
        if m >= 256:  # 256 x 512 pair tiles (group 0: as many as keep 64 MB of x)
            for group in (0, 8):
                out.append(("bf16", _lib.MusePlan(kernel=_lib.KERNEL_TC_WIDE, split=group)))
    if 16 < m <= 1024:
        # The pair GEMM with W as the A operand: all tokens (up to 256) or half of them a pair tile,
        # K split across as many pairs as fill one wave (and half that).
        pairs = sms // 2
        rpairs = (n + 255) // 256
        for t in sorted({min(256, (m + 15) // 16 * 16), min(256, ((m + 1) // 2 + 15) // 16 * 16)}):
            ptiles = rpairs * ((m + t - 1) // t)
            smax = min(pairs // ptiles, nkb, 64) if ptiles <= pairs else 1
            divisor = lambda lim: max(d for d in range(1, max(1, lim) + 1) if t % d == 0)  # the split divides T
            for s in sorted({divisor(smax), divisor(smax // 2)}):
                out.append(("bf16", _lib.MusePlan(kernel=_lib.KERNEL_TC_PAIRK, tile_n=t, split=s)))
            if -(-ptiles * nkb // pairs) <= nkb:  # stream-K: equal runs of at most one tile each
                out.append(("bf16", _lib.MusePlan(kernel=_lib.KERNEL_TC_PAIRK, tile_n=t, flags=_lib.FLAG_STREAMK)))
    if bnt <= 128:
        for stages, ctas in ((4, 2 * sms), (6, sms), (8, sms)):
            if bnt >= 128 and ctas > sms:
                continue
            out.append(("bf16", _lib.MusePlan(kernel=_lib.KERNEL_TC_STREAMK, tile_n=bnt, stages=stages, ctas=ctas)))
    return out


class ShapeBench:
    """R cold copies of one weight shape (BF16 and, when requested, 12-bit) and their inputs."""

    def __init__(self, n: int, k: int, m_max: int, twelve: bool, seed: int = 0):
        self.n, self.k = n, k
        copy_bytes = n * k * 2
        self.rot = max(2, min(12, math.ceil(3 * L2_BYTES / copy_bytes)))
        g = torch.Generator(device="cuda").manual_seed(seed)
        self.w = [(torch.randn((n, k), generator=g, device="cuda") * 0.02).to(torch.bfloat16) for _ in range(self.rot)]
        self.x = [torch.randn((m_max, k), generator=g, device="cuda").to(torch.bfloat16) for _ in range(self.rot)]
        self.y = [torch.empty((m_max, n), dtype=torch.bfloat16, device="cuda") for _ in range(self.rot)]
        st = torch.cuda.current_stream().cuda_stream
        self.tiles = []
        for w in self.w:
            t = torch.empty(_lib.tiles_bytes(n, k), dtype=torch.uint8, device="cuda")
            _lib.pack_tiles(w.data_ptr(), t.data_ptr(), n, k, st)
            self.tiles.append(t)
        self.scratch = torch.zeros(128 << 20, dtype=torch.uint8, device="cuda")
        self.enc = []
        if twelve and k % 512 == 0:
            from .submission import _Enc12Device
            for w in self.w:
                host = codec12.encode(w.cpu().view(torch.int16).numpy().view(np.uint16))
                self.enc.append(_Enc12Device(host, torch.device("cuda")))

    def launch(self, i: int, m: int, fmt: str, plan: _lib.MusePlan) -> None:
        j = i % self.rot
        st = torch.cuda.current_stream().cuda_stream
        if fmt == "12b" and plan.kernel in (_lib.KERNEL_TC_12B, _lib.KERNEL_GEMV_12T):
            _lib.proj_12b_tiles(self.enc[j].view(self.n), self.enc[j].tiles12.data_ptr(), self.x[j].data_ptr(),
                                self.y[j].data_ptr(), m, plan, st, self.scratch.data_ptr(), self.scratch.numel())
        elif fmt == "12b":
            _lib.proj_12b(self.enc[j].view(self.n), self.x[j].data_ptr(), self.y[j].data_ptr(), m, plan, st)
        elif plan.kernel in _lib.TILE_KERNELS:
            _lib.proj_bf16_tiles(self.x[j].data_ptr(), self.tiles[j].data_ptr(), self.y[j].data_ptr(), m, self.n,
                                 self.k, plan, st, self.scratch.data_ptr(), self.scratch.numel())
        else:
            _lib.proj_bf16(self.x[j].data_ptr(), self.w[j].data_ptr(), self.y[j].data_ptr(), m, self.n, self.k, plan, st)

    def check(self, m: int, fmt: str, plan: _lib.MusePlan) -> float:
        self.y[0].fill_(float("nan"))
        self.launch(0, m, fmt, plan)
        torch.cuda.synchronize()
        if _lib.device_error(torch.cuda.current_stream().cuda_stream):
            return float("inf")
        ref = (self.x[0][:m].float() @ self.w[0].float().T).to(torch.bfloat16).float()
        got = self.y[0][:m].float()
        if not torch.isfinite(got).all():
            return float("inf")
        return ((got - ref).norm() / ref.norm()).item()

    def time_us(self, m: int, fmt: str, plan: _lib.MusePlan, reps: int) -> tuple[float, float]:
        """(back-to-back, bracketed) microseconds per launch: `reps` launches timed as one batch
        (start/end events only; the event clock ticks coarsely, so batches time precisely), and
        the mean of per-launch event pairs."""
        for i in range(3):
            self.launch(i, m, fmt, plan)
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(int(4e6 + reps * 1e5))  # host runs ahead of the GPU: no launch gaps
        start.record()
        for i in range(reps):
            self.launch(i, m, fmt, plan)
        end.record()
        torch.cuda.synchronize()
        batch = start.elapsed_time(end) * 1e3 / reps
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
        torch.cuda._sleep(int(4e6 + reps * 1e5))
        for i, (a, b) in enumerate(evs):
            a.record()
            self.launch(i, m, fmt, plan)
            b.record()
        torch.cuda.synchronize()
        return batch, statistics.mean(a.elapsed_time(b) * 1e3 for a, b in evs)


    def one_call_us(self, m: int, fmt: str, plan: _lib.MusePlan, reps: int) -> float:
        """One launch timed as the reference's judge times a call (validate.py:124-147): captured in a
        CUDA graph, a 256 MB read to flush L2, then the replay between two events; the mean over `reps`
        (the event clock ticks in 2.048 us steps, which the replays' random phase resolves in a mean)."""
        if getattr(self, "flush", None) is None:
            self.flush = torch.ones(64 << 20, dtype=torch.float32, device="cuda")
        cur = torch.cuda.current_stream()
        side = torch.cuda.Stream()
        side.wait_stream(cur)
        with torch.cuda.stream(side):
            self.launch(0, m, fmt, plan)
            self.launch(0, m, fmt, plan)
        cur.wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.launch(0, m, fmt, plan)
        torch.cuda.synchronize()
        times = []
        for _ in range(reps):
            self.flush.sum()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(cur)
            g.replay()
            b.record(cur)
            torch.cuda.synchronize()
            times.append(a.elapsed_time(b) * 1e3)
        del g
        return statistics.fmean(times)

    def cublas_us(self, m: int, reps: int) -> float:
        """Back-to-back microseconds per call of torch's F.linear (cuBLAS) on the same rotating
        weights and inputs: the reference's scoring baseline (baseline.py:56-60, restated as
        F.linear in validate.py:97-105), timed as time_us times a batch. A comparator only."""
        import torch.nn.functional as F
        for i in range(3):
            F.linear(self.x[i % self.rot][:m], self.w[i % self.rot])
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(int(4e6 + reps * 1e5))
        start.record()
        for i in range(reps):
            F.linear(self.x[i % self.rot][:m], self.w[i % self.rot])
        end.record()
        torch.cuda.synchronize()
        return start.elapsed_time(end) * 1e3 / reps


def trace_plan(sb: "ShapeBench", m: int, fmt: str, plan: _lib.MusePlan, log, launches: int = 4) -> dict:
    """Runs the plan `launches` times back to back, each launch tracing into its own buffer, and
    summarises every launch on one clock: first CTA start, last CTA end, per-CTA prologue / main
    loop / epilogue medians. Consecutive launches overlapping (programmatic launch) shows up as a
    launch starting before the previous one ended."""
    cap = 4096
    bufs = [torch.zeros(cap * _lib.TRACE_RECORD_BYTES // 8, dtype=torch.int64, device="cuda") for _ in range(launches)]
    for i in range(3):
        sb.launch(i, m, fmt, plan)
    torch.cuda.synchronize()
    try:
        for i in range(launches):
            _lib.set_trace(bufs[i].data_ptr(), cap)
            sb.launch(3 + i, m, fmt, plan)
    finally:
        _lib.set_trace(0, 0)
    torch.cuda.synchronize()
    per, raws = [], []
    t_origin = None
    for b in bufs:
        rec = b.cpu().numpy().reshape(cap, 8)
        t = rec[:, :4].astype(np.int64)
        valid = t[:, 3] > 0
        t = t[valid]
        if t_origin is None:
            t_origin = t[:, 0].min()
        rel = (t - t_origin) / 1e3
        per.append({"ctas": int(valid.sum()), "first_start": round(float(rel[:, 0].min()), 3),
                    "last_start": round(float(rel[:, 0].max()), 3), "first_end": round(float(rel[:, 3].min()), 3),
                    "last_end": round(float(rel[:, 3].max()), 3),
                    "prologue": round(float(np.median(rel[:, 1] - rel[:, 0])), 3),
                    "main_med": round(float(np.median(rel[:, 2] - rel[:, 1])), 3),
                    "main_max": round(float(np.max(rel[:, 2] - rel[:, 1])), 3),
                    "tail_med": round(float(np.median(rel[:, 3] - rel[:, 2])), 3),
                    "tail_max": round(float(np.max(rel[:, 3] - rel[:, 2])), 3)})
        for c in range(6):  # kernel-specific marks: ns after the main loop's end
            w = rec[valid, 5 + c // 2].astype(np.uint64)
            v = (w >> np.uint64(32 * (c % 2))) & np.uint64(0xFFFFFFFF)
            if v.any():
                per[-1][f"mark{c + 1}_med"] = round(float(np.median(v.astype(np.float64))) / 1e3, 3)
        meta = rec[valid, 4].astype(np.uint64)
        raws.append({"t_us": rel.round(3).tolist(), "sm": (meta & 0xFFFFFFFF).astype(np.int64).tolist(),
                     "cta": ((meta >> 32) & 0xFFFFFFFF).astype(np.int64).tolist()})
    for i, p in enumerate(per):
        log(f"trace n={sb.n} k={sb.k} m={m} {plan.as_dict()['kernel']} flags={plan.flags} launch {i}: {json.dumps(p)}")
    return {"launches": per, "raw": raws}


def sweep_shape(n, k, ms, reps, sms, twelve, log, only=None, trace=False, extra_flags=0, kernels=None, one_call=0):
    sb = ShapeBench(n, k, max(ms), twelve)
    rows = []
    for m in ms:
        results = []
        cands = only if only is not None else candidates(m, n, k, sms, twelve and bool(sb.enc))
        if kernels:
            cands = [(f, p) for f, p in cands if p.as_dict()["kernel"] in kernels]
        if extra_flags:
            cands = [(f, _lib.MusePlan.from_dict({**p.as_dict(), "flags": p.flags | extra_flags})) for f, p in cands]
        for fmt, plan in cands:
            try:
                err = sb.check(m, fmt, plan)
            except _lib.MuseError as e:
                log(f"  n={n} k={k} m={m} {fmt} {plan.as_dict()}: {e}")
                continue
            if not err <= 1e-3:
                log(f"  n={n} k={k} m={m} {fmt} {plan.as_dict()}: WRONG rel {err:.3e}")
                continue
            med, mean = sb.time_us(m, fmt, plan, reps)
            one = sb.one_call_us(m, fmt, plan, one_call) if one_call else None
            if one is not None:
                log(f"  n={n} k={k} m={m} {fmt} {plan.as_dict()}: {med:.2f} us back to back, one call {one:.2f} us")
            tr = trace_plan(sb, m, fmt, plan, log) if trace else None
            wbytes = n * k * (1.5 if fmt == "12b" else 2)
            gbs = (wbytes + m * k * 2 + m * n * 2) / (med * 1e-6) / 1e9
            results.append({"fmt": fmt, "plan": plan.as_dict(), "us": med, "us_mean": mean, "gbs": gbs, "rel": err,
                            "one_call_us": one, "trace": tr})
        results.sort(key=lambda r: r["us"])
        best16 = next((r for r in results if r["fmt"] == "bf16"), None)
        cub = sb.cublas_us(m, reps)
        for r in results[:3]:
            log(f"n={n} k={k} m={m}: {r['us']:.2f} us {r['gbs']:.0f} GB/s {r['fmt']} {r['plan']}")
        log(f"n={n} k={k} m={m}: cuBLAS F.linear {cub:.2f} us")
        rows.append({"n": n, "k": k, "m": m, "best": results[0] if results else None, "best_bf16": best16,
                     "all": results, "cublas_us": cub})
    del sb
    torch.cuda.empty_cache()
    return rows


def table_entries(rows) -> list[dict]:
    """Dispatch rows from sweep results. The winner timed at M serves (previous timed M, M];
    neighbouring ranges with the same plan merge. Where the overall winner is 12-bit, the best
    BF16 plan gets a row too, for layers served without 12-bit planes. 12-bit rows come first."""
    by_shape: dict = {}
    for r in rows:
        by_shape.setdefault((r["n"], r["k"]), []).append(r)
    entries = []
    for (n, k), rs in sorted(by_shape.items()):
        rs.sort(key=lambda r: r["m"])
        for key in ("best", "best_bf16"):
            cur, prev_m = None, 0
            for r in rs:
                lo, hi, prev_m = prev_m + 1, r["m"], r["m"]
                b = r[key]
                if b is None or (key == "best_bf16" and r["best"] is not None and r["best"]["fmt"] == "bf16"):
                    cur = None
                    continue
                plan = {kk: v for kk, v in b["plan"].items() if v}
                cub = r.get("cublas_us")
                if cur is not None and cur["plan"] == plan and cur["weights"] == b["fmt"] and cur["m_hi"] == lo - 1:
                    cur["m_hi"] = hi
                    cur["us"][str(r["m"])] = round(b["us"], 3)
                    if cub is not None:
                        cur.setdefault("cublas_us", {})[str(r["m"])] = round(cub, 3)
                    continue
                cur = {"n": n, "k": k, "m_lo": lo, "m_hi": hi, "weights": b["fmt"], "plan": plan,
                       "us": {str(r["m"]): round(b["us"], 3)}}
                if cub is not None:
                    cur["cublas_us"] = {str(r["m"]): round(cub, 3)}
                entries.append(cur)
    entries.sort(key=lambda e: (e["n"], e["k"], 0 if e["weights"] == "12b" else 1, e["m_lo"]))
    merged = []
    for e in entries:
        p = merged[-1] if merged else None
        if (p is not None and (p["n"], p["k"], p["weights"]) == (e["n"], e["k"], e["weights"])
                and p["plan"] == e["plan"] and p["m_hi"] + 1 == e["m_lo"]):
            p["m_hi"] = e["m_hi"]
            p["us"].update(e["us"])
            if "cublas_us" in e:
                p.setdefault("cublas_us", {}).update(e["cublas_us"])
        else:
            merged.append(e)
    return merged


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", default="reference,baseline")
    ap.add_argument("--ms", default=",".join(map(str, DEFAULT_MS)))
    ap.add_argument("--reps", type=int, default=40)
    ap.add_argument("--no-12b", action="store_true")
    ap.add_argument("--out", default="sweep.json")
    ap.add_argument("--write-table", action="store_true")
    ap.add_argument("--merge", action="store_true",
                    help="with --write-table / --from-json: replace only the swept shapes' rows up to the largest swept M")
    ap.add_argument("--plan", default="", help='time only this plan, e.g. {"kernel": "tc_tile", "split": 3}')
    ap.add_argument("--trace", action="store_true", help="also record per-CTA timestamps of each plan")
    ap.add_argument("--flags", type=int, default=0, help="plan flags OR-ed into every candidate (2 = PDL)")
    ap.add_argument("--kernels", default="", help="comma-separated kernel names: time only their candidates")
    ap.add_argument("--one-call", type=int, default=0, metavar="REPS",
                    help="also time each candidate as one call the judge's way (graph replay after an L2 flush), mean of REPS")
    ap.add_argument("--from-json", default="", help="write the table from an earlier sweep's JSON (no GPU)")
    args = ap.parse_args()
    if args.from_json:
        with open(args.from_json) as f:
            done = json.load(f)
        write_table(done["rows"], done.get("device", "?"), print, args.merge, args.no_12b)
        return
    torch.backends.cuda.matmul.allow_tf32 = False
    only = None
    if args.plan:
        d = json.loads(args.plan)
        only = [("12b" if d.get("kernel") in ("gemv_12b", "tc_12b", "gemv_12t") else "bf16", _lib.MusePlan.from_dict(d))]
    shapes = []
    for s in args.shapes.split(","):
        if s == "reference":
            shapes += REFERENCE_SHAPES
        elif s == "baseline":
            shapes += BASELINE_SHAPES
        elif s == "mlp":
            shapes += MLP_SHARD_SHAPES
        elif "x" in s:
            a, b = s.split("x")
            shapes.append((int(a), int(b)))
    ms = [int(v) for v in args.ms.split(",")]
    sms = _lib.sm_count()
    lines = []

    def log(msg):
        print(msg, flush=True)
        lines.append(msg)

    t0 = time.time()
    rows = []
    for n, k in shapes:
        shape_ms = [m for m in ms if not (n == UNPOOL_SLICE and m > 8)]
        if not shape_ms:
            continue
        rows += sweep_shape(n, k, shape_ms, args.reps, sms, not args.no_12b, log, only, args.trace, args.flags,
                            set(args.kernels.split(",")) if args.kernels else None, args.one_call)
    os.makedirs(os.path.dirname(args.out) or ".", exist_ok=True)
    with open(args.out, "w") as f:
        json.dump({"device": torch.cuda.get_device_name(), "sms": sms, "rows": rows,
                   "seconds": time.time() - t0}, f)
    if args.write_table:
        write_table(rows, torch.cuda.get_device_name(), log, args.merge, args.no_12b)


def merge_entries(old: list, new: list, bf16_only: bool = False) -> list:
    """The committed table's rows with the swept ones replaced: for every (N, K) shape that `new`
    covers, the old rows for M up to the largest M `new` covers are dropped (a row reaching past it
    is cut to start above it) and `new`'s rows take their place; other shapes and larger M keep
    their rows, so a targeted re-sweep of a few shapes or of small M updates only those. With
    `bf16_only` (a sweep without 12-bit candidates) an old 12-bit row in the swept range stays if
    it beats the new BF16 row at every M both timed. Sorted by shape, format and M."""
    top: dict = {}
    for e in new:
        top[(e["n"], e["k"])] = max(top.get((e["n"], e["k"]), 0), e["m_hi"])

    def new_us(key, m):
        for e in new:
            if (e["n"], e["k"]) == key and e["m_lo"] <= m <= e["m_hi"] and str(m) in e["us"]:
                return e["us"][str(m)]
        return None

    kept = []
    for e in old:
        key = (e["n"], e["k"])
        if key not in top or e["m_lo"] > top[key]:
            kept.append(e)
            continue
        if bf16_only and e.get("weights") == "12b":
            pairs = [(t, new_us(key, int(m))) for m, t in e["us"].items() if int(m) <= top[key]]
            if pairs and all(u is not None and t < u for t, u in pairs):
                kept.append(e)
                continue
        if e["m_hi"] > top[key]:
            cut = {**e, "m_lo": top[key] + 1}
            for field in ("us", "cublas_us"):
                if field in e:
                    cut[field] = {m: t for m, t in e[field].items() if int(m) > top[key]}
            kept.append(cut)
    return sorted(kept + list(new), key=lambda e: (e["n"], e["k"], e.get("weights", "bf16"), e["m_lo"]))


def write_table(rows, device: str, log, merge: bool = False, bf16_only: bool = False) -> None:
    entries = table_entries(rows)
    if merge and os.path.exists(TABLE_PATH):
        with open(TABLE_PATH) as f:
            entries = merge_entries(json.load(f).get("entries", []), entries, bf16_only)
    table = {"generated_by": "python -m muse_bf16_proj_b200.sweep --write-table [--merge] (or --from-json of its output)",
             "device": device,
             "timing": ("us = mean per launch of back-to-back launches (programmatic launch), weights cold in L2; "
                        "cublas_us = torch F.linear (cuBLAS) timed the same way on the same weights and inputs"),
             "entries": entries}
    with open(TABLE_PATH, "w") as f:
        json.dump(table, f, indent=1)
    log(f"wrote {len(table['entries'])} rows to {TABLE_PATH}")


if __name__ == "__main__":
    main()
