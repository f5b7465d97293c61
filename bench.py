"""Benchmark: quantized GEMV sweep (BASELINE config 2 at its largest shape).

One step = one M=1 matrix-vector product over a 151936 x 2048 weight matrix in each
of the six swept GGUF formats (Q4_0, Q4_K, Q5_K, Q6_K, Q8_0, MXFP4) -- the decode
head shape of the baseline's MoE models.  Metric: algorithmic HBM GB/s
(sum over formats of N*row_bytes + K*4 + N*4, divided by the step time).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

value     device-resident (weights and x in HBM), CUDA events on the library stream.
e2e       through the reference-named C-ABI (quant_matmul_omp of combined_engine.so)
          with pinned HOST x/out: H2D of x and D2H of out inside the timed region
          (weights resident after their first use, as the reference's are loaded once).
roofline  the dominant kernel (Q8_0 GEMV) timed per launch with CUDA events.
cpu_baseline  the reference C engine (compiled from its own sources into oracle/_ref)
          on the host cores, on the same weights (MXFP4 re-encoded in the reference's
          own layout), with all host threads.
N > 1     independent per-GPU replicas (the GEMV does not shard; weak scaling).
Synthetic data: 4096 distinct weight rows ~ N(0, 0.02), quantized by each format's
GGUF rule, tiled to 151936 rows; x ~ N(0, 1).  Every matrix (165-331 MB) is larger
than the 126 MB L2, so no L2 flush is needed between steps.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

FORMATS = [("Q4_0", 2), ("Q4_K", 12), ("Q5_K", 13), ("Q6_K", 14), ("Q8_0", 8), ("MXFP4", 39)]
N_ROWS, K_COLS, DISTINCT = 151936, 2048, 4096
METRIC = "quant-GEMV HBM GB/s (M=1, 151936x2048, 6 GGUF formats)"
WORKLOAD = "quant-GEMV sweep Q4_0,Q4_K,Q5_K,Q6_K,Q8_0,MXFP4 at 151936x2048, M=1 (BASELINE config 2)"
BLOCK = {2: (32, 18), 12: (256, 144), 13: (256, 176), 14: (256, 210), 8: (32, 34), 39: (32, 17)}


def row_bytes(qt):
    be, bb = BLOCK[qt]
    return K_COLS // be * bb


def alg_bytes(qt, m=1):
    return N_ROWS * row_bytes(qt) + m * K_COLS * 4 + m * N_ROWS * 4


def make_weights(qt, seed=0, ref_layout=False):
    """bench-local synthetic weights: quantize DISTINCT rows, tile to N_ROWS.
    ref_layout re-encodes MXFP4 in the reference C decoder's own layout."""
    from mojollama_b200 import gguf_quant as Q
    rng = np.random.default_rng(seed * 1000 + qt)
    vals = (rng.standard_normal(DISTINCT * K_COLS) * 0.02).astype(np.float32)
    base = Q.quantize(Q.MXFP4_REF if (ref_layout and qt == 39) else qt, vals)
    reps = -(-N_ROWS // DISTINCT)
    w = np.tile(base, reps)[: N_ROWS * row_bytes(qt)]
    return np.ascontiguousarray(w)


class Clocks:
    """nvidia-smi sampler for the timed region."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = os.path.join(ROOT, "gpurun_out", f"clocks_{os.getpid()}.csv")

    def start(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index),
                 "--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        time.sleep(0.25)
        self.proc.terminate()
        self.proc.wait(timeout=5)
        self.f.close()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            p = [v.strip() for v in line.split(",")]
            if len(p) < 7:
                continue
            try:
                sm.append(float(p[0]))
                mx.append(float(p[1]))
            except ValueError:
                continue
            for n, v in zip(names, p[3:7]):
                if v.lower() == "active":
                    reasons.add(n)
        try:
            os.remove(self.path)
        except OSError:
            pass
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------------------ reference arm
def run_reference(args, rank, world):
    if rank != 0:
        return 0
    from oracle import formats as F
    from oracle import ref as R
    if not R.available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref not built (make -C oracle)"}))
        return 0
    eng = R.RefEngine()
    threads = os.cpu_count() or 1
    eng.set_num_threads(threads)
    ws = {}
    for name, qt in FORMATS:
        ws[qt] = make_weights(qt, ref_layout=True)
    x = np.random.default_rng(1).standard_normal(K_COLS).astype(np.float32)
    out = np.zeros(N_ROWS, np.float32)

    def step():
        for name, qt in FORMATS:
            eng.so.quant_matmul_omp(R.uptr(ws[qt]), R.fptr(x), R.fptr(out), N_ROWS, K_COLS, qt)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    gbs = sum(alg_bytes(qt) for _, qt in FORMATS) / dt / 1e9
    line = {"impl": "reference", "metric": METRIC, "value": round(gbs, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic", "config": {"workload": WORKLOAD, "global_batch": 1, "parallelism": "cpu"},
            "cpu_baseline": {"value": round(gbs, 2), "unit": "GB/s", "cores": threads, "kind": "reference",
                             "sample": "the full step (6 formats x 151936x2048 GEMV) per step"},
            "e2e": {"value": round(gbs, 2), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))
    return 0


def cpu_baseline_sample(seconds=12.0):
    """Reference C quant_matmul_omp on the host cores, bounded sample of the workload."""
    try:
        from oracle import formats as F
        from oracle import ref as R
        if not R.available():
            return {"value": None, "unit": "GB/s", "cores": 0, "kind": "reference",
                    "sample": "unavailable: oracle/_ref not built"}
        eng = R.RefEngine()
        threads = os.cpu_count() or 1
        eng.set_num_threads(threads)
        x = np.random.default_rng(1).standard_normal(K_COLS).astype(np.float32)
        out = np.zeros(N_ROWS, np.float32)
        total_b, total_t, reps = 0.0, 0.0, 0
        per = {}
        for name, qt in FORMATS:
            w = make_weights(qt, ref_layout=True)
            eng.so.quant_matmul_omp(R.uptr(w), R.fptr(x), R.fptr(out), N_ROWS, K_COLS, qt)   # warm
            t0 = time.perf_counter()
            n = 0
            while time.perf_counter() - t0 < seconds / len(FORMATS) or n < 2:
                eng.so.quant_matmul_omp(R.uptr(w), R.fptr(x), R.fptr(out), N_ROWS, K_COLS, qt)
                n += 1
            dt = time.perf_counter() - t0
            per[name] = round(alg_bytes(qt) * n / dt / 1e9, 2)
            total_b += alg_bytes(qt) * n
            total_t += dt
            reps += n
        return {"value": round(total_b / total_t / 1e9, 2), "unit": "GB/s", "cores": threads,
                "kind": "reference", "per_format": per,
                "sample": f"{reps} quant_matmul_omp calls over the 6 formats at 151936x2048 (~{seconds:.0f} s)"}
    except Exception as e:  # never let the baseline break the GPU line
        return {"value": None, "unit": "GB/s", "cores": 0, "kind": "reference", "sample": f"failed: {e}"}


# ------------------------------------------------------------------------------ our arm
def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from mojollama_b200 import core
    from mojollama_b200.kernels import load_kernels

    torch.cuda.set_device(local_rank)
    lib = core()
    assert lib.mlq_init(local_rank) == 0, lib.mlq_last_error_message()
    kern = load_kernels().kern
    stream = torch.cuda.Stream()
    lib.mlq_set_stream(ctypes.c_void_p(stream.cuda_stream))

    host_w = {qt: make_weights(qt) for _, qt in FORMATS}
    dev_w = {qt: torch.from_numpy(w).cuda() for qt, w in host_w.items()}
    x = torch.randn(K_COLS, generator=torch.Generator().manual_seed(1)).cuda()
    outs = {qt: torch.empty(N_ROWS, device="cuda") for _, qt in FORMATS}
    torch.cuda.synchronize()

    def step_dev(ev_pairs=None):
        for name, qt in FORMATS:
            if ev_pairs is not None and qt == 8:
                ev_pairs[-1][0].record(stream)
            rc = lib.mlq_matmul(ctypes.c_void_p(dev_w[qt].data_ptr()), qt, ctypes.c_void_p(x.data_ptr()),
                                ctypes.c_void_p(outs[qt].data_ptr()), N_ROWS, K_COLS, 1)
            if ev_pairs is not None and qt == 8:
                ev_pairs[-1][1].record(stream)
            if rc:
                raise RuntimeError(lib.mlq_last_error_message())

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(max(3, args.warmup)):
        step_dev()
    stream.synchronize()

    clocks = Clocks(local_rank)
    clocks.start()
    barrier()
    torch.cuda.synchronize()
    launches0 = lib.mlq_launch_count()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    q8_events = []
    start.record(stream)
    for _ in range(args.steps):
        q8_events.append((torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)))
        step_dev(q8_events)
    end.record(stream)
    stream.synchronize()
    barrier()
    torch.cuda.synchronize()
    launches = lib.mlq_launch_count() - launches0
    ms = start.elapsed_time(end)
    q8_ms = [a.elapsed_time(b) for a, b in q8_events]
    clk = clocks.stop()

    # e2e through the reference-named C-ABI with pinned host buffers
    hx = torch.empty(K_COLS, dtype=torch.float32, pin_memory=True)
    hx.copy_(x.cpu())
    hout = torch.empty(N_ROWS, dtype=torch.float32, pin_memory=True)
    hx_np, hout_np = hx.numpy(), hout.numpy()
    cf = ctypes.POINTER(ctypes.c_float)
    cu = ctypes.POINTER(ctypes.c_uint8)

    def step_e2e():
        for name, qt in FORMATS:
            kern.quant_matmul_omp(host_w[qt].ctypes.data_as(cu), hx_np.ctypes.data_as(cf),
                                  hout_np.ctypes.data_as(cf), N_ROWS, K_COLS, qt)

    for _ in range(max(3, args.warmup)):
        step_e2e()          # first call also makes each host weight resident
    barrier()
    torch.cuda.synchronize()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    for _ in range(args.steps):
        step_e2e()
    e_end.record(stream)
    stream.synchronize()
    e2e_ms = e_start.elapsed_time(e_end)

    # max over ranks
    t = torch.tensor([ms, e2e_ms, statistics.mean(q8_ms)], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms, q8_avg = (float(v) for v in t.tolist())

    step_bytes = sum(alg_bytes(qt) for _, qt in FORMATS)
    value = world * step_bytes * args.steps / (ms / 1e3) / 1e9
    e2e_value = world * step_bytes * args.steps / (e2e_ms / 1e3) / 1e9
    if rank != 0:
        return 0
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    hbm_peak = peaks.get("hbm_gbs", 6650.0)
    q8_bytes = alg_bytes(8)
    achieved = q8_bytes / (q8_avg / 1e3) / 1e9
    traffic = None
    tp = os.path.join(ROOT, "profiles", "gemv_q8_0_traffic.json")
    if os.path.exists(tp):
        try:
            traffic = json.load(open(tp)).get("bytes_per_launch")
        except Exception:
            traffic = None
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8-dp4a/fp32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "global_batch": world, "seq_len": 1,
                   "parallelism": f"replicas{world}" if world > 1 else "single",
                   "l2": "every weight matrix (165-331 MB) is larger than L2; no flush"},
        "per_format_gbs": None,
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s",
                "h2d_bytes_per_step": K_COLS * 4 * len(FORMATS), "d2h_bytes_per_step": N_ROWS * 4 * len(FORMATS),
                "api": "combined_engine.so quant_matmul_omp, pinned host x/out, resident weights"},
        "gpu_launches": int(launches),
        "roofline": {"bound": "hbm", "kernel": "k_gemv_q<Q8_0,1>", "achieved": round(achieved, 1),
                     "peak": hbm_peak, "unit": "GB/s", "frac": round(achieved / hbm_peak, 4),
                     "traffic": traffic, "peak_source": "measured" if peaks else "fallback"},
        "clocks": clk,
    }
    # per-format device GB/s (one extra timed pass, events around each launch)
    per = {}
    for name, qt in FORMATS:
        evs = []
        for _ in range(5):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            lib.mlq_matmul(ctypes.c_void_p(dev_w[qt].data_ptr()), qt, ctypes.c_void_p(x.data_ptr()),
                           ctypes.c_void_p(outs[qt].data_ptr()), N_ROWS, K_COLS, 1)
            b.record(stream)
            evs.append((a, b))
        stream.synchronize()
        per[name] = round(alg_bytes(qt) / (statistics.median(a.elapsed_time(b) for a, b in evs) / 1e3) / 1e9, 1)
    line["per_format_gbs"] = per
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_sample(args.cpu_seconds)
    print(json.dumps(line), flush=True)
    return 0


def run_profile_case(fmt: str, rows: int, launches: int = 3) -> int:
    """Small single-kernel case for `ncu --set full`: one format, `rows` x 2048, M=1,
    two warm-up launches then `launches` more.  Default 65536 rows keeps every matrix
    above the 126 MB L2 for Q8_0 (142 MB) and the whole run at a few hundred MB."""
    import torch
    from mojollama_b200 import core
    qt = dict(FORMATS)[fmt]
    lib = core()
    assert lib.mlq_init(0) == 0
    from mojollama_b200 import gguf_quant as Q
    rng = np.random.default_rng(qt)
    base = Q.quantize(qt, (rng.standard_normal(DISTINCT * K_COLS) * 0.02).astype(np.float32))
    w = np.tile(base, -(-rows // DISTINCT))[: rows * row_bytes(qt)]
    wd = torch.from_numpy(np.ascontiguousarray(w)).cuda()
    x = torch.randn(K_COLS, device="cuda")
    out = torch.empty(rows, device="cuda")
    lib.mlq_set_stream(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    for _ in range(2 + launches):
        rc = lib.mlq_matmul(ctypes.c_void_p(wd.data_ptr()), qt, ctypes.c_void_p(x.data_ptr()),
                            ctypes.c_void_p(out.data_ptr()), rows, K_COLS, 1)
        assert rc == 0, lib.mlq_last_error_message()
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": fmt, "rows": rows, "cols": K_COLS, "bytes_per_launch":
                      rows * row_bytes(qt) + K_COLS * 4 + rows * 4}))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--profile", default=None, help="run the small single-kernel ncu case for FORMAT")
    ap.add_argument("--profile-rows", type=int, default=65536)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.profile:
        return run_profile_case(args.profile, args.profile_rows)
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        return run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
