#!/usr/bin/env python
"""Throughput benchmark: series-forecasts/sec of the t0-alpha-shape quantized
forecast path on B200, N GPUs.

Workload (the box-wide sweep configuration, one context length per run):
8192 independent multivariate series in total, v ~ U{1..8} variates (seed
0), each variate a sum of 2-3 sinusoids + trend + N(0,0.2) noise with a 5%
NaN gap, context 2048 (p = 67 patches), horizon 96, random-init t0-alpha
weights exported to Q8_0 GGUF.  With N GPUs the batch is split into N
contiguous token-balanced shards of whole series (weights replicated), each
rank forecasts its shard, and the quantiles are all-gathered over NCCL
inside the timed step (strong scaling: total work fixed).  `--weak` instead
gives every rank its own 8192 series and no collective.  A step = one
forecast of the whole batch.

The default run also checks the timed step's output against the CPU oracle
on a sample of series (`parity`; the run exits non-zero when it is off),
times the oracle on the host cores (`cpu_baseline`, all threads and one
thread) and, on one GPU, adds the single-forecast latency and every size
of the two standalone GEMM configurations as `secondary` (each with its own
clock record).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--quant q8_0|q4_0]
                    [--ctx 2048] [--impl ours|reference] [--weak]

Under torchrun each rank drives one GPU; rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "series-forecasts/sec (t0-alpha-shape, quantized GEMMs resident as GGUF blocks)"
L2_FLUSH_BYTES = 256 << 20


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--quant", default="q8_0", choices=["q8_0", "q4_0"])
    ap.add_argument("--model", default="alpha", choices=["alpha", "beta"],
                    help="t0-alpha shape (default, the headline) or t0-beta shape (embed_dim 1024, head_dim 128, "
                         "21 quantiles); random-init weights either way")
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--series", type=int, default=8192)
    ap.add_argument("--horizon", type=int, default=96)
    ap.add_argument("--variates", default="1-8",
                    help="variates per series: a range lo-hi drawn uniformly (default 1-8, the box-wide sweep) "
                         "or a fixed count (3 with --series 256: the 256-trivariate-series configuration)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-sample", type=int, default=0, help="series per CPU-baseline step (0 = one per thread)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--strong", action="store_true",
                    help="(default) split one fixed set of series across the ranks, NCCL all-gather of the quantiles")
    ap.add_argument("--weak", action="store_true", help="every rank forecasts its own series, no collective")
    ap.add_argument("--no-secondary", action="store_true",
                    help="skip the single-forecast latency and standalone GEMM lines of the default run")
    ap.add_argument("--parity-series", type=int, default=0,
                    help="series checked against the oracle (0 = the CPU-baseline sample, at least 8)")
    ap.add_argument("--workload", default="forecast", choices=["forecast", "single", "gemm", "swiglu"],
                    help="forecast: the multi-series headline (default); single: one-series latency (cfg 1); "
                         "gemm: standalone Q8_0 dequant-GEMM N=3072 K=1024 (cfg 2); swiglu: standalone Q4_0 "
                         "SwiGLU F=4096 K=1024 N2=1024 (cfg 3).  The extra workloads print one line per case.")
    a = ap.parse_args()
    a.strong = not a.weak
    return a


def variates(args):
    lo, _, hi = args.variates.partition("-")
    return (int(lo), int(hi)) if hi else int(lo)


def workload(args, seed):
    from t0_web_b200 import synthetic as S
    ctx, nv = S.multiseries(args.series, args.ctx, seed=seed, n_variates=variates(args))
    return ctx, nv


def config_block(args, nv, world):
    p = (args.ctx + (32 - args.ctx % 32) % 32 + (args.horizon + 31) // 32 * 32) // 32
    rows = int(nv.sum())
    per = "in total" if args.strong else "per GPU"
    par = ("series-sharded, weights replicated, NCCL all-gather of quantiles" if args.strong else
           "independent series per GPU, weights replicated, no data-path collective")
    return {
        "workload": (f"{args.series} multivariate series {per} ("
                     f"{'v~U{' + args.variates.replace('-', '..') + '}' if '-' in args.variates else 'v=' + args.variates}"
                     f", seed {args.seed}"
                     f"{'' if args.strong else ' + rank'}), ctx {args.ctx}, horizon {args.horizon}, "
                     f"t0-{args.model} shape random-init weights as {args.quant.upper()} GGUF"),
        "series": args.series, "series_total": args.series * (1 if args.strong else world),
        "rows": rows, "patches_per_row": p, "tokens": rows * p,
        "ctx": args.ctx, "horizon": args.horizon, "quant": args.quant,
        "parallelism": f"dp{world} ({par})",
        "l2": "inputs larger than L2 (>=38 MB contexts + GBs of activations per step) and a 256 MB "
              "buffer write between timed steps",
    }


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def load_oracle():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    return O


def oracle_sample(omodel, ctx, nv, horizon, n_series, threads, steps=1, warmup=0):
    """Times the oracle (plain-C t0-core restatement) on the first n_series
    series of the workload with `threads` host threads; returns (series/s,
    per-step seconds, the last step's quantiles [rows, horizon, nq])."""
    import numpy as np
    rows = int(np.sum(nv[:n_series]))
    c, v = ctx[:rows], nv[:n_series]
    for _ in range(warmup):
        omodel.forecast_multiseries(c, v, horizon, threads=threads)
    times, out = [], None
    for _ in range(steps):
        t0 = time.perf_counter()
        out = omodel.forecast_multiseries(c, v, horizon, threads=threads)
        times.append(time.perf_counter() - t0)
    return n_series / (sum(times) / len(times)), times, out


def gpu_uuid(device):
    import torch
    try:
        return str(torch.cuda.get_device_properties(device).uuid).lower().replace("gpu-", "")
    except Exception:
        return ""


class ClockSampler:
    """nvidia-smi clock samples every 200 ms, kept only for the GPUs the run
    uses (matched by UUID; by index if the UUIDs are unavailable)."""
    FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuids=(), indices=()):
        self.proc = None
        self.uuids = {u for u in uuids if u}
        self.indices = set(indices)
        self.path = os.path.join("/tmp", f"t0b_clocks_{os.getpid()}_{id(self)}.csv")

    def _lines(self):
        try:
            with open(self.path) as f:
                return sum(1 for _ in f)
        except OSError:
            return 0

    def _wait_lines(self, more_than, timeout_s):
        t_end = time.time() + timeout_s
        while self._lines() <= more_than and time.time() < t_end and self.proc.poll() is None:
            time.sleep(0.01)

    def start(self):
        """Starts sampling and returns once the first sample is written, so a
        short timed region that follows is bracketed by samples."""
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
            return self
        self._wait_lines(0, 5.0)
        return self

    def stop(self):
        if not self.proc:
            return None
        self._wait_lines(self._lines(), 0.5)  # one more sample after the timed region
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 10:
                try:
                    rows.append((int(f[0]), f[1].lower().replace("gpu-", ""), float(f[2]), float(f[3]),
                                 f[6], f[7], f[8], f[9]))
                except ValueError:
                    pass
        try:
            os.remove(self.path)
        except OSError:
            pass
        mine = [r for r in rows if r[1] in self.uuids] if self.uuids else []
        how = "uuid"
        if not mine:
            mine = [r for r in rows if r[0] in self.indices] if self.indices else rows
            how = "index" if self.indices else "all"
        if not mine:
            return None
        mx = max(r[3] for r in mine)
        loaded = [r[2] for r in mine if r[2] > 0.3 * mx] or [r[2] for r in mine]
        reasons = set()
        for r in mine:
            for name, val in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"), r[4:]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(mine), "gpus": sorted({r[0] for r in mine}), "matched_by": how}


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            j = json.load(f)
        return float(j["bf16_tflops_sustained"]), float(j["hbm_gbs"]), "measured"
    except Exception:
        return 1400.0, 6650.0, "fallback"


def model_cfg(args):
    from t0_web_b200 import synthetic as S
    return S.BETA if getattr(args, "model", "alpha") == "beta" else S.ALPHA


def committed_traffic(quant, model="alpha"):
    """DRAM bytes per gemm_tc launch from the committed ncu summary (t0-alpha
    shapes only), if any."""
    if model != "alpha":
        return None
    try:
        with open(os.path.join(ROOT, "profiles", "gemm_tc_traffic.json")) as f:
            return json.load(f).get(quant)
    except Exception:
        return None


def parity_series(nv, ranges, per_rank):
    """Indices of the series checked against the oracle: the first
    `per_rank` series of every rank's shard."""
    out = []
    for lo, hi in ranges:
        out.extend(range(lo, min(hi, lo + per_rank)))
    return sorted(set(out))


def rows_of(nv, series):
    import numpy as np
    cum = np.concatenate([[0], np.cumsum(np.asarray(nv, np.int64))])
    return np.concatenate([np.arange(cum[s], cum[s + 1]) for s in series]) if series else np.zeros(0, np.int64)


# ----------------------------------------------------------------- our arm
def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    from t0_web_b200 import gguf, sharded, synthetic as S, t0_fast

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))

    cfg = model_cfg(args)
    weights = S.random_weights(cfg, seed=0)
    gbytes = gguf.export_gguf(weights, cfg, args.quant)
    del weights
    # strong (default): one set of series split across the ranks; weak: every rank its own
    ctx, nv = workload(args, args.seed if args.strong else args.seed + rank)
    engine = t0_fast.Engine(local)
    model = t0_fast.load_model_from_gguf(engine, gbytes)
    # one explicit stream for the library, the timing events and the collective
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    model.set_stream(stream.cuda_stream)

    if args.strong:
        row_ranges = sharded.shard_rows(nv, world)
        ser_ranges = sharded.balanced_split(nv, world)
    else:
        row_ranges = [(0, int(nv.sum()))] * world
        ser_ranges = [(0, len(nv))] * world
    r0, r1 = row_ranges[rank]
    s0, s1 = ser_ranges[rank]
    rows_per_rank = [b - a for a, b in row_ranges]
    nq = model.n_quantiles
    ctx_shard = np.ascontiguousarray(ctx[r0:r1])
    nv_shard = np.ascontiguousarray(nv[s0:s1])
    ctx_dev = torch.from_numpy(ctx_shard).cuda()
    out_dev = torch.empty((r1 - r0, args.horizon, nq), device="cuda")
    flush = torch.empty(L2_FLUSH_BYTES // 4, device="cuda")
    gather = args.strong and world > 1
    ag_evs = []

    def step(record_gather=False):
        if s1 > s0:
            t0_fast.forecast_multiseries_device(model, ctx_dev, nv_shard, args.ctx, args.horizon, out_dev)
        if gather:
            if record_gather:
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
            g = sharded.gather_outputs(out_dev, rows_per_rank)
            if record_gather:
                b.record(stream)
                ag_evs.append((a, b))
            return g
        return out_dev

    # ---- secondary workloads (one GPU): single-forecast latency, small-M
    # GEMMs; run first, while the GPU is not yet power-capped by the long step
    secondary = None
    if rank == 0 and world == 1 and not args.no_secondary and args.model == "alpha":
        secondary = {"single_forecast": run_single(args, engine=engine, model=model, emit=False)}
        for wl in ("gemm", "swiglu"):  # every size of the standalone configurations
            for line in run_standalone(args, workload=wl, engine=engine, emit=False):
                secondary[f"{wl}_M{line['config_M']}"] = line

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    uuids = [gpu_uuid(local)]
    if world > 1:
        allu = [None] * world
        dist.all_gather_object(allu, uuids[0])
        uuids = allu
        dist.barrier()

    sampler = ClockSampler(uuids, range(world)).start() if rank == 0 else None
    model.profile(True)
    launches0 = model.launch_count()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    for a, b in evs:
        flush.zero_()  # L2 flush, outside the timed bracket
        a.record(stream)
        full = step(record_gather=True)
        b.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    total_ms = sum(a.elapsed_time(b) for a, b in evs)
    ag_ms = sum(a.elapsed_time(b) for a, b in ag_evs)
    prof = model.profile_read()
    launches = model.launch_count() - launches0
    model.profile(False)
    clocks = sampler.stop() if sampler else None
    passes = prof.get("prep", {}).get("launches", 0) / args.steps  # one prep launch per pass
    series_total = args.series * (1 if args.strong else world)
    t = torch.tensor([total_ms, float(launches), ag_ms, passes], dtype=torch.float64, device="cuda")
    per_rank = None
    if world > 1:
        tm = t[:1].clone()
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
        tl = t[1:2].clone()
        dist.all_reduce(tl, op=dist.ReduceOp.SUM)
        pr = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(pr, t)
        per_rank = [{"rank": i, "ms_per_step": float(x[0]) / args.steps, "allgather_ms_per_step": float(x[2]) / args.steps,
                     "passes_per_step": float(x[3]), "rows": rows_per_rank[i]} for i, x in enumerate(pr)]
        total_ms, launches = float(tm.item()), int(tl.item())
    ms_per_step = total_ms / args.steps
    value = series_total / (ms_per_step / 1e3)
    full_host = full.cpu().numpy() if rank == 0 else None  # the last timed step's (gathered) output

    # ---- end to end through the public host API (H2D and D2H inside) ----
    e2e = None
    if not args.no_e2e:
        if gather:
            ctx_pin = torch.from_numpy(ctx_shard).pin_memory()
            full_pin = torch.empty((sum(rows_per_rank), args.horizon, nq), dtype=torch.float32).pin_memory() \
                if rank == 0 else None

        def e2e_step():
            if gather:
                # sharded: every rank copies its contexts up from pinned host
                # memory and forecasts into device memory, the quantiles are
                # all-gathered on the devices, and the rank that returns the
                # result (0) copies the gathered quantiles down once
                ctx_dev.copy_(ctx_pin, non_blocking=True)
                g = step()
                if rank == 0:
                    full_pin.copy_(g, non_blocking=True)
                stream.synchronize()
                return full_pin
            # one GPU (or --weak): the host-buffer entry point, copies inside
            out = t0_fast.forecast_multiseries(engine, model, ctx_shard, nv_shard, args.ctx, args.horizon) \
                if s1 > s0 else np.zeros((0, args.horizon, nq), np.float32)
            return out
        e2e_step()
        times = []
        for _ in range(args.steps):
            if world > 1:
                dist.barrier()
            t0 = time.perf_counter()
            e2e_step()
            times.append(time.perf_counter() - t0)
        et = torch.tensor([sum(times), float(ctx_shard.nbytes), float(ctx_shard.shape[0] * args.horizon * nq * 4)],
                          dtype=torch.float64, device="cuda")
        if world > 1:
            e_max = et[:1].clone()
            dist.all_reduce(e_max, op=dist.ReduceOp.MAX)
            e_sum = et[1:].clone()
            dist.all_reduce(e_sum, op=dist.ReduceOp.SUM)
            et = torch.cat([e_max, e_sum])
        e_ms = float(et[0].item()) * 1e3 / args.steps
        h2d = int(et[1].item())  # every rank copies its own contexts in
        d2h = int(et[2].item())  # its quantiles out (sharded: the gathered quantiles, once, on rank 0)
        e2e = {"value": series_total / (e_ms / 1e3), "unit": "series/s", "ms_per_step": e_ms,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}

    # ---- roofline of the dominant kernel (tcgen05 dequant GEMM) ----
    peak_tf, peak_gbs, peak_kind = measured_peaks()
    g = prof.get("gemm_tc", {})
    roofline = None
    if g.get("launches"):
        per_launch_ms = g["total_ms"] / g["launches"]
        achieved = g["flops"] / (g["total_ms"] / 1e3) / 1e12
        tr = committed_traffic(args.quant, args.model)
        if tr:  # per-token DRAM bytes of one launch (ncu) x this run's tokens per launch
            n_gemm = 4 * model.info.num_layers
            tok_per_launch = (int(nv_shard.sum()) * config_block(args, nv, world)["patches_per_row"] * n_gemm
                              * args.steps / g["launches"])
            tr = tr["dram_bytes_per_token_per_launch"] * tok_per_launch
        roofline = {"kernel": "gemm_q_tc_pair_kernel", "bound": "tensor", "achieved": achieved, "peak": peak_tf,
                    "unit": "TFLOP/s", "frac": achieved / peak_tf,
                    "peak_kind": f"{peak_kind} bf16 sustained (dense cuBLAS)",
                    "traffic": tr, "avg_launch_ms": per_launch_ms,
                    "flops_per_launch": g["flops"] / g["launches"],
                    "share_of_step": g["total_ms"] / max(total_ms, 1e-9),
                    "issued_frac": 3.0 * achieved / peak_tf,
                    "issued_note": "f32-class accuracy takes 3 f16 MMAs per useful multiply-add (Ah.Wh + Ah.Wl + "
                                   "Al.Wh); issued_frac counts them, frac counts useful flops only",
                    "epilogue_note": "the launches also do the residual add + split of x*g + row sums of squares "
                                     "(wO, mlp.2), QK-norm gains + RoPE + split planes (TIME-layer wQKV) and SwiGLU "
                                     "(mlp.0); only the GEMM flops are counted"}
    breakdown = {k: {"launches": v["launches"], "ms": round(v["total_ms"], 3)} for k, v in prof.items()
                 if v["launches"]}

    # ---- CPU oracle: baseline timing and the parity sample ----
    cpu, parity = None, None
    if rank == 0:
        O = load_oracle()
        om = O.OracleModel(gbytes)
        th = cpu_threads()
        want = args.parity_series or 8
        ref, series = None, None
        if world == 1 and not args.no_cpu:
            n = args.cpu_sample or th
            rate, _, ref_n = oracle_sample(om, ctx, nv, args.horizon, n, th, steps=1)
            rate1, _, _ = oracle_sample(om, ctx, nv, args.horizon, 1, 1, steps=1)
            cpu = {"value": rate, "unit": "series/s", "cores": th, "kind": "port",
                   "sample": f"first {n} series of the same workload, one series per thread, oracle/t0_oracle.c",
                   "one_thread": {"value": rate1, "unit": "series/s", "cores": 1,
                                  "sample": "first series of the same workload, one thread (the reference engine "
                                            "is single-threaded)"}}
            if n >= want:  # the timed CPU sample doubles as the parity sample
                series, ref = list(range(n)), ref_n
        if ref is None:
            per = max(1, -(-want // world))
            # strong: the first series of every rank's shard (the output is gathered);
            # weak: rank 0's own series
            series = parity_series(nv, ser_ranges if args.strong else [(0, len(nv))], per)
            ref = om.forecast_multiseries(ctx[rows_of(nv, series)], nv[series], args.horizon, threads=th)
        rows = rows_of(nv, series)
        got = full_host[rows]
        d = np.abs(got.astype(np.float64) - ref.astype(np.float64))
        mx = float(np.max(d))
        # t0-alpha: 1e-3 max-abs (the north star's bound).  t0-beta's random-init
        # 21-level head drives the upper quantiles to ~1e6-1e7, beyond f32 for
        # an absolute 1e-3, so there the bound is 1e-3 of max(1, |reference|)
        rel = float(np.max(d / np.maximum(1.0, np.abs(ref.astype(np.float64)))))
        beta = args.model == "beta"
        parity = {"max_abs": mx, "max_rel_of_max1": rel, "tol": 1e-3,
                  "bound": "max |got - ref| / max(1, |ref|)" if beta else "max |got - ref|",
                  "series": len(series), "rows": int(len(rows)),
                  "ok": bool(np.isfinite(got).all() and (rel if beta else mx) <= 1e-3),
                  "checked": "the last timed step's output (gathered over the ranks) against the CPU oracle on "
                             "the same GGUF and contexts"}
    if world > 1:
        dist.barrier()  # ranks wait while rank 0 runs the oracle

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "series/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
                "scaling": "strong" if args.strong else "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic", "config": config_block(args, nv, world), "e2e": e2e, "roofline": roofline,
                "cpu_baseline": cpu, "parity": parity, "clocks": clocks, "gpu_launches": launches,
                "passes_per_step": passes, "allgather_ms_per_step": (ag_ms / args.steps) if gather else None,
                "per_rank": per_rank, "kernels": breakdown, "secondary": secondary,
                "arith": "GEMMs: split-f16 (3 MMAs, exact weight split) on tcgen05 with f32 TMEM accumulation; "
                         "attention, norms, scaler in f32"}
        print(json.dumps(line), flush=True)
    model.close()
    engine.close()
    if world > 1:
        dist.destroy_process_group()
    if rank == 0 and parity is not None and not parity["ok"]:
        sys.exit(3)


# ----------------------------------------------------- secondary workloads
def run_single(args, engine=None, model=None, emit=True):
    """cfg 1: one univariate series, ctx 512, horizon 96 (M = 19 tokens per
    GEMM: the small-M kernel).  value = median ms per forecast through the
    host API; roofline = that kernel's weight bytes per launch / its mean
    device time (HBM bound)."""
    import numpy as np

    from t0_web_b200 import gguf, synthetic as S, t0_fast
    quant = args.quant
    own = model is None
    if own:
        cfg = model_cfg(args)
        weights = S.random_weights(cfg, seed=0)
        gbytes = gguf.export_gguf(weights, cfg, quant)
        del weights
        engine = t0_fast.Engine(0)
        model = t0_fast.load_model_from_gguf(engine, gbytes)
    ctx = S.sine_context(512, seed=0)

    def timed(n):
        for _ in range(max(args.warmup, 3)):
            t0_fast.forecast(engine, model, ctx, 1, 512, 96)
        out = []
        for _ in range(n):
            t0 = time.perf_counter()
            t0_fast.forecast(engine, model, ctx, 1, 512, 96)
            out.append((time.perf_counter() - t0) * 1e3)
        return out

    nsteps = max(args.steps, 400)  # about 0.3 s, so the 200 ms clock sampler sees it
    sampler = ClockSampler([gpu_uuid(0)], [0]).start()
    times = timed(nsteps)                 # default: passes replayed from CUDA graphs
    clocks = sampler.stop()
    model.use_graphs(False)
    eager = timed(nsteps)                 # one host launch per kernel
    model.use_graphs(True)
    model.profile(True)                   # per-kernel device times (events, no graphs)
    timed(nsteps)
    prof = model.profile_read()
    model.profile(False)
    peak_tf, peak_gbs, kind = measured_peaks()
    g = prof.get("gemm_small", {})
    roof = None
    if g.get("launches"):
        gbs = g["bytes"] / (g["total_ms"] / 1e3) / 1e9
        roof = {"kernel": "gemm_q_small_kernel", "bound": "hbm", "achieved": gbs, "peak": peak_gbs, "unit": "GB/s",
                "frac": gbs / peak_gbs, "peak_kind": f"{kind} HBM copy",
                "avg_launch_us": 1e3 * g["total_ms"] / g["launches"],
                "bytes_per_launch": g["bytes"] / g["launches"]}
    n = nsteps
    dev_ms = sum(v["total_ms"] for v in prof.values()) / n
    line = {"metric": "single forecast latency (ctx 512, h 96, univariate)", "value": float(np.median(times)),
            "unit": "ms", "higher_is_better": False, "n_gpus": 1, "steps": n, "dtype": "f32",
            "data": "synthetic", "config": {"workload": f"cfg1 sine context, t0-{args.model} random-init {quant}",
                                            "tokens_per_gemm": 19},
            "eager_launch_ms": float(np.median(eager)),
            "device_ms_per_forecast": dev_ms,
            "chain_weight_GBps": (model.quantizable_gpu_bytes() / (float(np.median(times)) / 1e3) / 1e9),
            "kernels": {k: {"launches": v["launches"] // n, "ms": round(v["total_ms"] / n, 4)}
                        for k, v in prof.items() if v["launches"]},
            "roofline": roof, "clocks": clocks}
    if own:
        model.close()
        engine.close()
    if emit:
        print(json.dumps(line), flush=True)
    return line


def run_standalone(args, workload=None, cases=None, engine=None, emit=True):
    """cfg 2 / cfg 3 through the resident-weight C ABI (t0b_qmatrix_gemm /
    t0b_qmatrix_swiglu), device buffers.  Timing protocol: distinct weight
    copies are rotated so that one pass over them is >= 4x the 126 MB L2
    (weights never hit in L2), L calls are captured in one CUDA graph, and
    the median of 20 graph replays (CUDA events on the capture stream) / L is
    the time per call.  A call includes the split of x into f16 planes."""
    import ctypes as C

    import numpy as np
    import torch

    from t0_web_b200 import gguf, t0_fast
    from t0_web_b200._lib import Q4_0, Q8_0, check, lib, ptr
    workload = workload or args.workload
    own = engine is None
    if own:
        engine = t0_fast.Engine(0)
    dev = torch.device("cuda:0")
    st = torch.cuda.Stream()
    sp = C.c_void_p(st.cuda_stream)
    peak_tf, peak_gbs, kind = measured_peaks()
    rng = np.random.default_rng(0)
    L2 = 126 << 20

    def handle(wd, N, K):
        h = C.c_void_p()
        check(lib().t0b_qmatrix_create(engine.handle, qt, ptr(wd), N, K, C.byref(h)))
        return h

    if workload == "gemm":
        N, K, qt = 3072, 1024, Q8_0
        w = rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)
        wb = torch.from_numpy(gguf.quantize(w, qt)).to(dev)
        wbytes = wb.numel()
        all_cases = [16, 256, 4096, 65536]
    else:
        F, K, N2, qt = 4096, 1024, 1024, Q4_0
        w0 = rng.standard_normal((2 * F, K), dtype=np.float32) * np.float32(0.02)
        w2 = rng.standard_normal((N2, F), dtype=np.float32) * np.float32(0.02)
        w0b = torch.from_numpy(gguf.quantize(w0, qt)).to(dev)
        w2b = torch.from_numpy(gguf.quantize(w2, qt)).to(dev)
        wbytes = w0b.numel() + w2b.numel()
        all_cases = [16, 1024, 65536]
    ncopy = int(np.ceil(4 * L2 / wbytes))
    if workload == "gemm":
        copies = [wb.clone() for _ in range(ncopy)]
        hs = [handle(c, N, K) for c in copies]
    else:
        copies = [(w0b.clone(), w2b.clone()) for _ in range(ncopy)]
        hs = [(handle(a, 2 * F, K), handle(b, N2, F)) for a, b in copies]
    lines = []
    for M in (cases or all_cases):
        x = torch.randn((M, K), device=dev)
        if workload == "gemm":
            y = torch.empty((M, N), device=dev)
            flops = 2.0 * M * N * K
            nbytes = wbytes + 4.0 * M * K + 4.0 * M * N

            def call(i):
                check(lib().t0b_qmatrix_gemm(hs[i % ncopy], ptr(x), M, None, ptr(y), sp))
        else:
            z = torch.empty((M, F), device=dev)
            y = torch.empty((M, N2), device=dev)
            flops = 2.0 * M * 2 * F * K + 2.0 * M * N2 * F
            # gate/up reads x, writes z (f32) and its f16 split; down reads the split, writes y
            nbytes = wbytes + 4.0 * M * K + 8.0 * M * F + 4.0 * M * F + 4.0 * M * N2

            def call(i):
                q0, q2 = hs[i % ncopy]
                check(lib().t0b_qmatrix_swiglu(q0, q2, ptr(x), M, None, None, ptr(z), ptr(y), sp))
        # per-call work >= the whole rotation: L calls cover every copy at least once
        per_call = nbytes
        ncalls = max(ncopy, int(np.ceil(4 * L2 / per_call)))
        ncalls = min(ncalls, 400)
        with torch.cuda.stream(st):
            for i in range(ncopy):  # grows the scratch, warms every handle
                call(i)
        st.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st, capture_error_mode="relaxed"):
            for i in range(ncalls):
                call(i)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        sampler = ClockSampler([gpu_uuid(0)], [0]).start()
        evs = []
        for _ in range(20):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(st)
            with torch.cuda.stream(st):
                g.replay()
            b.record(st)
            evs.append((a, b))
        torch.cuda.synchronize()
        clocks = sampler.stop()
        for h in hs:
            for q in (h if isinstance(h, tuple) else (h,)):
                check(lib().t0b_qmatrix_sync(q, None))
        ms = float(np.median([a.elapsed_time(b) for a, b in evs])) / ncalls
        del g
        tf = flops / (ms / 1e3) / 1e12
        gbs = nbytes / (ms / 1e3) / 1e9
        small = M < 128
        name = "Q8_0 dequant-GEMM N=3072 K=1024" if workload == "gemm" else \
            "Q4_0 SwiGLU MLP F=4096 K=1024 N2=1024 (gate/up + fused SiLU, down)"
        roof = ({"bound": "hbm", "achieved": gbs, "peak": peak_gbs, "unit": "GB/s", "frac": gbs / peak_gbs,
                 "peak_kind": f"{kind} HBM copy"} if small else
                {"bound": "tensor", "achieved": tf, "peak": peak_tf, "unit": "TFLOP/s", "frac": tf / peak_tf,
                 "peak_kind": f"{kind} bf16 (sustained)"})
        line = {"metric": f"{name}, M={M}", "config_M": M, "value": tf, "unit": "TFLOP/s (useful)", "ms_per_call": ms,
                "achieved_GBps": gbs, "algorithmic_bytes": nbytes, "higher_is_better": True, "n_gpus": 1,
                "dtype": "f32-class (split-f16)", "data": "synthetic N(0,0.02) weights, N(0,1) activations",
                "roofline": roof, "path": "tcgen05" if not small else "mma.sync small-M", "clocks": clocks,
                "timing": f"{ncalls} calls per CUDA graph over {ncopy} rotated weight copies "
                          f"({ncopy * wbytes / 2**20:.0f} MiB), median of 20 replays; a call = the "
                          "GEMM(s) on f32 x (GEMM: split into f16 planes inside the small-M kernel, one split pass "
                          "before the tensor-core kernel; SwiGLU: one split pass, then the two GEMMs)"}
        lines.append(line)
        if emit:
            print(json.dumps(line), flush=True)
    for h in hs:
        for q in (h if isinstance(h, tuple) else (h,)):
            lib().t0b_qmatrix_destroy(q)
    del copies
    torch.cuda.empty_cache()
    if own:
        engine.close()
    return lines


# ----------------------------------------------------------- reference arm
def run_reference(args):
    """The reference's CPU path for this workload: t0-core (Rust) cannot be
    built here, so its plain-C restatement (oracle/t0_oracle.c) runs on the
    host cores.  Nothing of the product library is loaded: the GGUF file is
    written by the oracle's own export_gguf and the contexts come from the
    pure-numpy generator."""
    rank = int(os.environ.get("RANK", 0))
    if rank != 0:
        return
    from t0_web_b200 import synthetic as S
    O = load_oracle()
    cfg = model_cfg(args)
    weights = S.random_weights(cfg, seed=0)
    gbytes = O.export_gguf(weights, cfg, args.quant)
    del weights
    ctx, nv = workload(args, args.seed)
    om = O.OracleModel(gbytes)
    th = cpu_threads()
    n = args.cpu_sample or th
    rate, times, _ = oracle_sample(om, ctx, nv, args.horizon, n, th, steps=args.steps, warmup=args.warmup)
    rate1, _, _ = oracle_sample(om, ctx, nv, args.horizon, 1, 1, steps=1)
    ms = 1e3 * sum(times) / len(times)
    line = {"metric": METRIC, "value": rate, "unit": "series/s", "n_gpus": int(os.environ.get("WORLD_SIZE", 1)),
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong" if args.strong else "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference", "config": config_block(args, nv, 1),
            "cpu_baseline": {"value": rate, "unit": "series/s", "cores": th, "kind": "port",
                             "sample": f"first {n} series of the workload per step, one series per thread; the "
                                       "reference (Rust t0-core) cannot be built here, so its plain-C "
                                       "restatement oracle/t0_oracle.c is timed",
                             "one_thread": {"value": rate1, "unit": "series/s", "cores": 1,
                                            "sample": "first series of the workload, one thread"}},
            "e2e": {"value": rate, "unit": "series/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    a = parse()
    if a.impl == "reference":
        run_reference(a)
    elif a.workload == "single":
        run_single(a)
    elif a.workload in ("gemm", "swiglu"):
        run_standalone(a)
    else:
        run_ours(a)
