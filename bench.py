"""Benchmark: quantized GEMV sweep (benchmark config 2 at its largest shape).

One step = one M=1 matrix-vector product over a 151936 x 2048 weight matrix in each
of the six swept GGUF formats (Q4_0, Q4_K, Q5_K, Q6_K, Q8_0, MXFP4) -- the decode
head shape of the baseline's MoE models.  Metric: algorithmic HBM GB/s
(sum over formats of N*row_bytes + K*4 + N*4, divided by the step time).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

value     device-resident (weights and x in HBM), CUDA events on the library stream.
e2e       through the reference-named C-ABI (quant_matmul_omp of combined_engine.so)
          with pinned HOST x/out: H2D of x and D2H of out inside the timed region
          (weights resident after their first use, as the reference's are loaded once).
roofline  the dominant kernel (the format whose GEMV takes the largest share of the step),
          each launch timed with CUDA events inside the timed region.
decode    config 1 (TinyLlama-1.1B shape, Q8_0, B=4) through batch_forward: tok/s device
          resident and end to end, with the reference C engine's batch_forward on the host
          cores as its CPU baseline (N = 1 only), and the logits of all 48 positions checked
          against the oracle (greedy tokens where the top-2 margin exceeds 1e-2).
qwen3moe  config 3 (Qwen3-30B-A3B shape, Q4_K_M, 48 layers, 128 experts top-8) through
          batch_forward at B = 1 and 16: decode tok/s, bytes per step and achieved bandwidth,
          end to end through the reference-named entry, the reference C ops on the host cores.
gptoss    config 4 (GPT-OSS-20B shape: bf16 attention alternating full / 128-token windows,
          32 MXFP4 experts top-4, 16-token pages) through batch_forward at B = 1, 16, 64.
hybrid    config 5 (hybrid [3 SSM + 1 GQA] x 10, 256 MXFP4 experts) through
          qwen36_batch_forward at B = 10; N > 1: one independent replica per GPU.
moe_ep    config 3's MoE FFN stack (48 layers, 128 experts top-8) with the experts split over
          the N GPUs and NCCL all-to-all dispatch/combine: tok/s (weak scaling), with the
          expert-parallel layer checked against the same layer on one GPU.
sweep     config 2 in full (6 formats x 4 shapes x M in {1, 4, 16, 64, 256}), one row per case.
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
# the kernel each format's M=1 GEMV runs (mojollama_b200/csrc/gemv.cu, gemv_mxf4_tc.cu)
KERNEL_OF = {"MXFP4": "k_gemv_mxf4_tc (tcgen05.mma kind::mxf4, UE8M0 block scales)"}
N_ROWS, K_COLS, DISTINCT = 151936, 2048, 4096
METRIC = "quant-GEMV HBM GB/s (M=1, 151936x2048, 6 GGUF formats)"
WORKLOAD = "quant-GEMV sweep Q4_0,Q4_K,Q5_K,Q6_K,Q8_0,MXFP4 at 151936x2048, M=1 (config 2)"
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
    """nvidia-smi sampler for the timed region (CSV in a temporary directory).

    start() returns once the first sample row exists (the sampler takes a few hundred ms
    to start), so samples cover the timed region that follows; `busy` (optional) keeps
    the GPU loaded while waiting, so the clocks seen are the clocks under load."""

    def __init__(self, index):
        import tempfile
        self.index = index
        self.proc = None
        self.path = os.path.join(tempfile.gettempdir(), f"mlq_clocks_{os.getpid()}_{index}.csv")

    def _rows(self):
        try:
            return sum(1 for line in open(self.path) if line.strip())
        except OSError:
            return 0

    def wait_first(self, busy=None, limit_s=3.0):
        t0 = time.perf_counter()
        while self.proc and self._rows() < 1 and time.perf_counter() - t0 < limit_s:
            if busy:
                busy()
            else:
                time.sleep(0.02)

    def start(self, busy=None):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index),
                 "--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        self.wait_first(busy)

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        n0 = self._rows()
        t0 = time.perf_counter()
        while self._rows() <= n0 and time.perf_counter() - t0 < 1.0:   # one sample after the region
            time.sleep(0.02)
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


def our_config(world):
    """the workload description both arms print (the reference arm runs the same workload
    on the host cores)"""
    return {"workload": WORKLOAD, "global_batch": world, "seq_len": 1,
            "parallelism": f"replicas{world}" if world > 1 else "single",
            "l2": "every weight matrix (165-331 MB) is larger than L2; no flush"}


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
            "data": "synthetic", "config": our_config(world),
            "cpu_baseline": {"value": round(gbs, 2), "unit": "GB/s", "cores": threads, "kind": "reference",
                             "sample": "the full step (6 formats x 151936x2048 GEMV) per step"},
            "e2e": {"value": round(gbs, 2), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))
    return 0


def gemv_traffic(fmt):
    """DRAM bytes (read + write) per full 151936 x 2048 launch of the M=1 GEMV of `fmt`,
    from the committed ncu summary profiles/gemv_traffic.md (rows `| FMT | ... | bytes |`),
    or None when that format has not been captured."""
    path = os.path.join(ROOT, "profiles", "gemv_traffic.md")
    try:
        for line in open(path):
            cells = [c.strip() for c in line.strip().strip("|").split("|")]
            if len(cells) >= 2 and cells[0] == fmt and cells[-1].replace(".", "").isdigit():
                return int(float(cells[-1]))
    except OSError:
        pass
    return None


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

    def step_dev(ev=None, only=None):
        """one step; ev: {qt: [(start, end), ...]} gets a pair of events around each launch
        (of format `only` alone when given)"""
        for name, qt in FORMATS:
            if ev is not None and (only is None or qt == only):
                pair = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                ev.setdefault(qt, []).append(pair)
                pair[0].record(stream)
            rc = lib.mlq_matmul(ctypes.c_void_p(dev_w[qt].data_ptr()), qt, ctypes.c_void_p(x.data_ptr()),
                                ctypes.c_void_p(outs[qt].data_ptr()), N_ROWS, K_COLS, 1)
            if ev is not None and (only is None or qt == only):
                pair[1].record(stream)
            if rc:
                raise RuntimeError(lib.mlq_last_error_message())

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(max(3, args.warmup)):
        step_dev()
    stream.synchronize()
    # untimed pass: every launch timed, to find the dominant kernel (largest share of a step)
    pre = {}
    for _ in range(3):
        step_dev(pre)
    stream.synchronize()
    pre_ms = {qt: statistics.mean(a.elapsed_time(b) for a, b in pairs) for qt, pairs in pre.items()}
    dom_name, dom_qt = max(FORMATS, key=lambda f: pre_ms[f[1]])

    clocks = Clocks(local_rank)
    clocks.start(busy=lambda: (step_dev(), stream.synchronize()))
    barrier()
    torch.cuda.synchronize()
    launches0 = lib.mlq_launch_count()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    fmt_events = {}
    start.record(stream)
    for _ in range(args.steps):
        step_dev(fmt_events, only=dom_qt)   # events around the dominant kernel's launches only
    end.record(stream)
    stream.synchronize()
    barrier()
    torch.cuda.synchronize()
    launches = lib.mlq_launch_count() - launches0
    ms = start.elapsed_time(end)
    dom_ms = statistics.mean(a.elapsed_time(b) for a, b in fmt_events[dom_qt])
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

    # the same calls with pageable numpy x/out: the reference Python's own call shape
    # (x staged through the library's arena by a copy, out copied back after the kernel)
    px = np.ascontiguousarray(hx_np.copy())
    pout = np.zeros(N_ROWS, np.float32)

    def step_e2e_pageable():
        for name, qt in FORMATS:
            kern.quant_matmul_omp(host_w[qt].ctypes.data_as(cu), px.ctypes.data_as(cf),
                                  pout.ctypes.data_as(cf), N_ROWS, K_COLS, qt)

    for _ in range(max(3, args.warmup)):
        step_e2e_pageable()
    barrier()
    torch.cuda.synchronize()
    p_start, p_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p_start.record(stream)
    for _ in range(args.steps):
        step_e2e_pageable()
    p_end.record(stream)
    stream.synchronize()
    e2e_pageable_ms = p_start.elapsed_time(p_end)
    assert lib.mlq_last_error() == 0, lib.mlq_last_error_message()

    # max over ranks
    t = torch.tensor([ms, e2e_ms, dom_ms, e2e_pageable_ms], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms, dom_ms, e2e_pageable_ms = (float(v) for v in t.tolist())

    step_bytes = sum(alg_bytes(qt) for _, qt in FORMATS)
    value = world * step_bytes * args.steps / (ms / 1e3) / 1e9
    e2e_value = world * step_bytes * args.steps / (e2e_ms / 1e3) / 1e9
    hyb = None
    if not args.no_hybrid:
        # config 5 as independent replicas: every rank runs its own, the slowest one counts
        hyb = run_hybrid(torch, lib, stream, rank, world)
        ht = torch.tensor([hyb["dec_ms"], hyb["pre_ms"]], device="cuda")
        if world > 1:
            dist.all_reduce(ht, op=dist.ReduceOp.MAX)
        hyb["dec_ms"], hyb["pre_ms"] = (float(v) for v in ht.tolist())
    if rank != 0:
        if not args.no_moe_ep:
            run_moe_ep(torch, lib, rank, world)   # every rank takes part in the collectives
        return 0
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    hbm_peak = peaks.get("hbm_gbs", 6650.0)
    # the dominant kernel (from the untimed pass), timed per launch inside the timed region
    achieved = alg_bytes(dom_qt) / (dom_ms / 1e3) / 1e9
    traffic = gemv_traffic(dom_name)
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8 dp4a (Q4_0/K-quants/Q8_0), e2m1 x ue8m0 tcgen05 (MXFP4); fp32 accumulate", "data": "synthetic",
        "config": our_config(world),
        "per_format_gbs": None,
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s",
                "h2d_bytes_per_step": K_COLS * 4 * len(FORMATS), "d2h_bytes_per_step": N_ROWS * 4 * len(FORMATS),
                "api": "combined_engine.so quant_matmul_omp, pinned host x/out, resident weights; x copied in, "
                       "out written into the pinned buffer by the GEMV kernel (d2h bytes cross PCIe in the kernel)",
                "pageable": {"value": round(world * step_bytes * args.steps / (e2e_pageable_ms / 1e3) / 1e9, 2),
                             "unit": "GB/s",
                             "api": "the same calls with pageable numpy x/out (the reference Python's call shape): "
                                    "x staged by a copy, out copied back after the kernel"}},
        "gpu_launches": int(launches),
        "roofline": {"bound": "hbm", "kernel": KERNEL_OF.get(dom_name, f"k_gemv_q1<{dom_name}>") + " (M=1 GEMV)",
                     "achieved": round(achieved, 1),
                     "peak": hbm_peak, "unit": "GB/s", "frac": round(achieved / hbm_peak, 4),
                     "traffic": traffic, "algorithmic_bytes": alg_bytes(dom_qt),
                     "share_of_step": round(pre_ms[dom_qt] / sum(pre_ms.values()), 3),
                     "peak_source": "measured" if peaks else "fallback"},
        "clocks": clk,
    }
    # per-format device GB/s from the untimed per-launch pass
    line["per_format_gbs"] = {name: round(alg_bytes(qt) / (pre_ms[qt] / 1e3) / 1e9, 1) for name, qt in FORMATS}
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_sample(args.cpu_seconds)
    if not args.no_decode and world == 1:
        line["decode"] = run_decode(torch, lib, stream, with_cpu=not args.no_cpu_baseline,
                                    cpu_seconds=args.cpu_seconds, with_parity=not args.no_parity)
    if hyb is not None:
        line["hybrid"] = hybrid_line(hyb, world)
    if not args.no_sweep and world == 1:
        # config 2 in full: one compact row per case, [format, N, K, M, us, GB/s, TFLOP/s]
        sw = sweep_cases(torch, lib, stream, SWEEP_M)
        line["sweep"] = {"metric": sw["metric"], "columns": ["fmt", "N", "K", "M", "us", "gbs", "tflops"],
                         "cases": [[c["fmt"], c["N"], c["K"], c["M"], c["us"], c["gbs"], c["tflops"]]
                                   for c in sw["cases"]]}
    if not args.no_gptoss and world == 1:
        line["gptoss"] = run_gptoss(torch, lib, stream)
    if not args.no_qwen3moe and world == 1:
        line["qwen3moe"] = run_qwen3moe(torch, lib, stream, with_cpu=not args.no_cpu_baseline,
                                        cpu_seconds=args.cpu_seconds)
    if not args.no_moe_ep:
        line["moe_ep"] = run_moe_ep(torch, lib, rank, world)
    print(json.dumps(line), flush=True)
    return 0


def run_decode_profile(args):
    """Small case for an ncu launch list of decode steps: the config-1 model, B = 4,
    `--profile-steps` batch_forward calls at positions 0.. (weights ~1.1 GB in HBM)."""
    import torch
    from mojollama_b200 import core
    lib = core()
    assert lib.mlq_init(0) == 0
    stream = torch.cuda.Stream()
    lib.mlq_set_stream(ctypes.c_void_p(stream.cuda_stream))
    b, keep, caches = build_tinyllama(torch, lib, 64)
    d_logits = torch.empty(TL["B"] * TL["V"], device="cuda")
    d_tok = torch.zeros(TL["B"], dtype=torch.int32, device="cuda")
    b.bc.logits = ctypes.cast(ctypes.c_void_p(d_logits.data_ptr()), ctypes.POINTER(ctypes.c_float))
    l0 = lib.mlq_launch_count()
    for _ in range(args.profile_steps):
        rc = lib.mlq_batch_forward(ctypes.byref(b.bc), ctypes.c_void_p(d_tok.data_ptr()), TL["B"], None)
        assert rc == 0, lib.mlq_last_error_message()
    stream.synchronize()
    print(json.dumps({"decode_profile_steps": args.profile_steps,
                      "launches_per_step": (lib.mlq_launch_count() - l0) // args.profile_steps}))
    for kv in caches:
        kv.free()
    return 0


# ------------------------------------------------------------------------------ MoE expert parallelism
# Config 3's MoE FFN: 48 layers, d_model 2048, 128 experts, softmax top-8 with
# renormalised weights, expert FFN 768, gate/up Q4_K and down Q6_K; the experts are split
# over the ranks (expert parallelism), the router replicated.  Tokens per rank fixed (weak
# scaling); each layer runs on the same N(0,1) token rows so the routing stays the one of
# the N(0,1)-scaled router (values are synthetic; the expert blocks are random bytes with
# small fp16 scales).
MOE = dict(L=48, E=128, k=8, N=2048, FF=768, gq=12, uq=12, dq=14)


def _random_kquant(torch, qt, n_blocks, gen):
    """random K-quant blocks on the device with a small fp16 super-block scale (1/1024) and
    dmin 0: finite, bounded weights for timing"""
    bb = {12: 144, 14: 210}[qt]
    w = torch.randint(0, 256, (n_blocks, bb), dtype=torch.uint8, device="cuda", generator=gen)
    if qt == 12:
        w[:, 0], w[:, 1], w[:, 2], w[:, 3] = 0x00, 0x14, 0x00, 0x00
    else:
        w[:, 208], w[:, 209] = 0x00, 0x14
    return w.reshape(-1)


def run_moe_ep(torch, lib, rank, world, tokens=16, steps=5, warmup=3, layers=None, with_parity=True, use_graph=True):
    import torch.distributed as dist
    from mojollama_b200.ep import EPMoELayer, row_bytes as rbytes
    # the library's kernels, the NCCL exchanges and the timing events all on torch's
    # current stream: the exchanges then follow the dispatch kernels, and the events
    # bracket the device work (not just its issue)
    lib.mlq_set_stream(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    c = dict(MOE)
    L = layers or c["L"]
    E, k, N, FF = c["E"], c["k"], c["N"], c["FF"]
    el = E // world
    gen = torch.Generator(device="cuda").manual_seed(1234 + rank)
    rgen = torch.Generator(device="cuda").manual_seed(99)   # same router on every rank
    from mojollama_b200.ep import expert_slice
    layer_objs = []
    exp_bytes = FF * rbytes(c["gq"], N) * 2 + N * rbytes(c["dq"], FF)
    full0 = None
    for li in range(L):
        router = torch.randn(E, N, device="cuda", generator=rgen) * 0.02
        if li == 0 and with_parity:
            # layer 0: every expert from one seed shared by the ranks, so that each rank can
            # also run the whole layer alone (all E experts resident) as the parity check
            g0 = torch.Generator(device="cuda").manual_seed(4321)
            full0 = [_random_kquant(torch, c["gq"], E * FF * N // 256, g0),
                     _random_kquant(torch, c["uq"], E * FF * N // 256, g0),
                     _random_kquant(torch, c["dq"], E * N * FF // 256, g0), router]
            g, u, d = (expert_slice(t, rank, world, E) for t in full0[:3])
        else:
            g = _random_kquant(torch, c["gq"], el * FF * N // 256, gen)
            u = _random_kquant(torch, c["uq"], el * FF * N // 256, gen)
            d = _random_kquant(torch, c["dq"], el * N * FF // 256, gen)
        layer_objs.append(EPMoELayer(rank, world, E, k, N, FF, c["gq"], c["uq"], c["dq"], g, u, d, router,
                                     renorm=True, max_tokens=tokens))
    x = torch.randn(tokens, N, device="cuda", generator=torch.Generator(device="cuda").manual_seed(7 + rank))

    def step():
        y = x
        for lay in layer_objs:
            y = lay.forward(x, residual=x)
        return y

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    # The step issues no host synchronisation (fixed-capacity exchanges), so it is captured
    # whole -- kernels and NCCL all-to-alls -- into one CUDA graph and replayed; the library
    # launches on the capture stream while capturing.  Eager timing if capture is refused.
    graph, graph_err = None, None
    if use_graph:
        try:
            g = torch.cuda.CUDAGraph()
            cap = torch.cuda.Stream()
            cap.wait_stream(torch.cuda.current_stream())
            # bound before the capture starts: rebinding inside it would synchronise the old stream
            lib.mlq_set_stream(ctypes.c_void_p(cap.cuda_stream))
            with torch.cuda.graph(g, stream=cap):
                g_out = step()
            lib.mlq_set_stream(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
            graph = g
            graph.replay()
            torch.cuda.synchronize()
        except Exception as e:   # keep the eager path
            graph_err = f"{type(e).__name__}: {e}"[:200]
            graph = None
            lib.mlq_set_stream(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
            torch.cuda.synchronize()
    ok = torch.tensor([0 if graph is None else 1], device="cuda")
    if world > 1:   # every rank takes the same path (the collectives must match)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if graph is not None and int(ok.item()) == 0:
        graph = None
    if world > 1:
        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    h0 = time.perf_counter()
    for _ in range(steps):
        if graph is not None:
            graph.replay()
            out = g_out
        else:
            out = step()
    host_ms = (time.perf_counter() - h0) * 1e3 / steps   # host time to issue one step
    b.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = torch.tensor([a.elapsed_time(b)], device="cuda")
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    t = float(ms.item()) / steps
    finite = bool(torch.isfinite(out).all().item())
    parity = None
    if full0 is not None:
        # expert-parallel layer 0 against the same layer with every expert on this rank
        # (world 1: no exchange) on the same tokens: the dispatch and combine move rows
        # without arithmetic, so the two must agree bit for bit
        alone = EPMoELayer(0, 1, E, k, N, FF, c["gq"], c["uq"], c["dq"], full0[0], full0[1], full0[2], full0[3],
                           renorm=True, max_tokens=tokens)
        y_ep = layer_objs[0].forward(x, residual=x)
        y_1 = alone.forward(x, residual=x)
        torch.cuda.synchronize()
        num = float(torch.linalg.vector_norm((y_ep - y_1).double()).item())
        den = float(torch.linalg.vector_norm(y_1.double()).item())
        res = torch.tensor([num / max(den, 1e-30), 0.0 if torch.equal(y_ep, y_1) else 1.0], device="cuda")
        if world > 1:
            dist.all_reduce(res, op=dist.ReduceOp.MAX)
        parity = {"check": "expert-parallel layer 0 vs the same layer with all experts on one GPU, same tokens, "
                           "every rank (max over ranks; eager)",
                  "ep_parity_rel_l2": float(res[0].item()), "dispatch_combine_bit_exact": res[1].item() == 0.0,
                  "tolerance": 1e-3, "ok": float(res[0].item()) <= 1e-3}
        del alone, full0
    used_graph = graph is not None
    if graph is not None:
        del graph, g_out   # a graph holding NCCL work is released before the process group goes
        torch.cuda.synchronize()
    return {"workload": f"config-3 MoE FFN stack: {L} layers, {E} experts top-{k} (renormalised), FF {FF}, "
                        f"Q4_K gate/up + Q6_K down, experts split over {world} GPU(s), fixed-capacity NCCL "
                        f"all-to-all (no host synchronisation in a step)",
            "tokens_per_rank": tokens, "tok_s": round(world * tokens / (t / 1e3), 1), "ms_per_step": round(t, 3),
            "expert_bytes_per_rank": L * el * exp_bytes, "scaling": "weak", "outputs_finite": finite,
            "cuda_graph": used_graph, **({"graph_error": graph_err} if graph_err else {}),
            "parity": parity,
            "host_issue_ms_per_step": round(host_ms, 3)}


# ------------------------------------------------------------------------------ config-3 whole model
# Qwen3-30B-A3B shape in Q4_K_M through batch_forward: 48 layers, d_model 2048, 32 / 4 heads
# of 128, 128 experts top-8 (FF 768; gate/up Q4_K, down Q6_K), router F32, attention Q4_K
# with V in Q6_K, output head 151936 x 2048 Q6_K, vocab 151936.  Prompt 128 tokens, then
# 64 decode steps, B = 1 and 16.  The batch engine's step (cengine_batch_instr.c:1233-1493)
# has no QK-RMSNorm and routes with moe_ffn's rule (no renormalisation); neither changes
# the bytes a step reads.  Synthetic weights: random K-quant blocks with small fp16 scales
# (finite, bounded values), router N(0, 1/N) so that its logits are ~N(0, 1).
Q3 = dict(L=48, N=2048, NH=32, NKH=4, HD=128, V=151936, E=128, k=8, M=768, eps=1e-6, prompt=128, gen=64)


def _kq_bytes(qt, rows, cols):
    be, bb = {12: (256, 144), 14: (256, 210), 8: (32, 34)}[qt]
    return rows * cols // be * bb


def qwen3moe_step_bytes(B, pos):
    """Algorithmic HBM bytes of one decode step: attention and router weights of every
    layer, the experts the step's tokens select (expected number of distinct experts under
    near-uniform routing, E (1 - (1 - k/E)^B)), the head, the embedding rows and the K/V rows
    read and written."""
    c = Q3
    N, inner, kv = c["N"], c["NH"] * c["HD"], c["NKH"] * c["HD"]
    attn = _kq_bytes(12, inner, N) + _kq_bytes(12, kv, N) + _kq_bytes(14, kv, N) + _kq_bytes(12, N, inner)
    router = c["E"] * N * 4
    expert = 2 * _kq_bytes(12, c["M"], N) + _kq_bytes(14, N, c["M"])
    distinct = c["E"] * (1 - (1 - c["k"] / c["E"]) ** B)
    head = _kq_bytes(14, c["V"], N)
    kv_bytes = B * c["L"] * 2 * kv * 4 * (pos + 2)
    return int(c["L"] * (attn + router + distinct * expert) + head + kv_bytes + B * (N * 4 + c["V"] * 4)), distinct


def build_qwen3moe(torch, lib, layers=None):
    from mojollama_b200 import bc as BCm
    c = Q3
    L, N, NH, NKH, HD, V, E, M = layers or c["L"], c["N"], c["NH"], c["NKH"], c["HD"], c["V"], c["E"], c["M"]
    inner, kv = NH * HD, NKH * HD
    g = torch.Generator(device="cuda").manual_seed(3)
    keep = []

    def kq(qt, rows, cols):
        t = _random_kquant(torch, qt, rows * cols // 256, g)
        keep.append(t)
        return t.data_ptr()

    b = BCm.BCBuilder()
    bc = b.bc
    bc.L, bc.N, bc.NH, bc.NKH, bc.HD, bc.FF, bc.V, bc.eps, bc.nc = L, N, NH, NKH, HD, 0, V, c["eps"], N
    for nm, qt, r, k in (("wQ", 12, inner, N), ("wK", 12, kv, N), ("wV", 14, kv, N), ("wO", 12, N, inner)):
        b.layers(nm, [kq(qt, r, k) for _ in range(L)])
    for f, v in (("nQ", inner), ("nK", kv), ("nV", kv), ("nO", N)):
        b.ints(f, [v] * L)
    for f, v in (("q_quant", 12), ("k_quant", 12), ("v_quant", 14), ("o_quant", 12)):
        b.ints(f, [v] * L)
    ones = torch.ones(N, device="cuda")
    keep.append(ones)
    b.layers("wAN", [ones.data_ptr()] * L)
    b.layers("wFN", [ones.data_ptr()] * L)
    routers = [torch.randn(E * N, generator=g, device="cuda") * (1.0 / np.sqrt(N)) for _ in range(L)]
    keep.extend(routers)
    b.layers("w_gate_inp", [r.data_ptr() for r in routers])
    b.layers("w_gate_exps", [kq(12, E * M, N) for _ in range(L)])
    b.layers("w_up_exps", [kq(12, E * M, N) for _ in range(L)])
    b.layers("w_down_exps", [kq(14, E * N, M) for _ in range(L)])
    bc.n_experts, bc.n_experts_per_tok, bc.moe_intermediate = E, c["k"], M
    bc.gate_exp_quant, bc.up_exp_quant, bc.down_exp_quant = 12, 12, 14
    emb = torch.randn(V * N, generator=g, device="cuda") * 0.02
    keep.append(emb)
    bc.emb, bc.emb_quant = emb.data_ptr(), 0
    bc.onw = ones.data_ptr()
    bc.wOut = kq(14, V, N)
    bc.outNR, bc.outNC, bc.outQuant = V, N, 14
    max_ctx = c["prompt"] + c["gen"] + 8
    j = np.arange(HD // 2)
    theta = np.arange(max_ctx)[:, None] / np.power(1e6, 2.0 * j / HD)   # rope_freq_base 1e6 (Qwen3)
    b.ptr("cos_table", np.cos(theta).astype(np.float32))
    b.ptr("sin_table", np.sin(theta).astype(np.float32))
    bc.max_ctx, bc.rope_dim = max_ctx, HD
    torch.cuda.synchronize()
    return b, keep


def run_qwen3moe(torch, lib, stream, with_cpu=True, cpu_seconds=10.0):
    """Config 3 decode through the library's batch_forward with on-device greedy sampling
    (mlq_batch_forward_sample: tokens never leave the device), per batch size: tok/s,
    bytes per step and achieved bandwidth, and end to end through the reference-named
    batch_forward of cengine_batch_instr.so with host tokens and host logits."""
    from mojollama_b200.serving import PagedKV
    from mojollama_b200.kernels import load_kernels
    c = Q3
    V, P, G = c["V"], c["prompt"], c["gen"]
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    hbm = peaks.get("hbm_gbs", 6650.0)
    prev = lib.mlq_get_stream()
    lib.mlq_set_stream(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    b, keep = build_qwen3moe(torch, lib)
    lib.mlq_set_stream(ctypes.c_void_p(prev))
    ce = load_kernels().cengine
    out = {"workload": "Qwen3-30B-A3B shape, Q4_K_M (Q4_K + Q6_K attn_v / ffn_down / output), 48 layers, "
                       "128 experts top-8, 128-token prompt then 64 greedy decode steps, through batch_forward "
                       "(config 3)", "batches": {}}
    for B in (1, 16):
        kvs = [PagedKV(c["L"], c["NKH"], c["HD"], 64, (P + G) // 64 + 2) for _ in range(B)]
        b.kv_array([k.block for k in kvs])
        d_logits = torch.empty(B * V, device="cuda")
        b.bc.logits = ctypes.cast(ctypes.c_void_p(d_logits.data_ptr()), ctypes.POINTER(ctypes.c_float))
        prompts = torch.from_numpy(np.random.default_rng(B).integers(0, V, (P, B)).astype(np.int32)).cuda()
        d_tok = torch.empty(B, dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()

        def fwd_sample(t):
            rc = lib.mlq_batch_forward_sample(ctypes.byref(b.bc), ctypes.c_void_p(d_tok.data_ptr()), B, None,
                                              ctypes.c_float(0.0), 0, t, ctypes.c_void_p(d_tok.data_ptr()))
            if rc:
                raise RuntimeError(lib.mlq_last_error_message())

        evs = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        with torch.cuda.stream(stream):
            evs[0].record(stream)
            for t in range(P):
                d_tok.copy_(prompts[t])
                fwd_sample(t)
            evs[1].record(stream)
            l0 = lib.mlq_launch_count()
            for t in range(G):
                fwd_sample(P + t)       # the sampled tokens feed the next step in place
            evs[2].record(stream)
        stream.synchronize()
        launches = (lib.mlq_launch_count() - l0) // G
        pre_ms, dec_ms = evs[0].elapsed_time(evs[1]), evs[1].elapsed_time(evs[2])
        sb = [qwen3moe_step_bytes(B, P + t) for t in range(G)]
        step_bytes = sum(x[0] for x in sb) / G
        ms = dec_ms / G
        # end to end: the reference's call shape (host tokens, host logits), 8 steps
        for k in kvs:
            k.block.seq_len[0] = P     # continue from the prompt (the positions already hold K/V rows)
        h_logits = np.zeros(B * V, np.float32)
        b.bc.logits = h_logits.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
        tok = np.zeros(B, np.int32)
        n_e2e = 8
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(n_e2e):
            ce.batch_forward(ctypes.byref(b.bc), tok.ctypes.data, B, None)
            tok = np.argmax(h_logits.reshape(B, V), axis=1).astype(np.int32)
        e2e_ms = (time.perf_counter() - t0) * 1e3 / n_e2e
        assert lib.mlq_last_error() == 0, lib.mlq_last_error_message()
        achieved = step_bytes / (ms / 1e3) / 1e9
        out["batches"][str(B)] = {
            "tok_s": round(B * G / (dec_ms / 1e3), 1), "ms_per_step": round(ms, 3),
            "prefill_tok_s": round(B * P / (pre_ms / 1e3), 1), "launches_per_step": int(launches),
            "e2e_tok_s": round(B / (e2e_ms / 1e3), 1), "e2e_ms_per_step": round(e2e_ms, 3),
            "e2e_io": {"h2d_bytes_per_step": B * 4, "d2h_bytes_per_step": B * V * 4},
            "roofline": {"bound": "hbm", "bytes_per_step": int(step_bytes),
                         "expected_distinct_experts_per_layer": round(sb[0][1], 1),
                         "achieved_gbs": round(achieved, 1), "peak": hbm, "frac": round(achieved / hbm, 4)}}
        for k in kvs:
            k.free()
        del d_logits
    if with_cpu:
        out["cpu_baseline"] = qwen3moe_cpu_baseline(torch, b, keep, cpu_seconds)
    del keep
    torch.cuda.empty_cache()
    return out


def qwen3moe_cpu_baseline(torch, b, keep, seconds):
    """The reference C engine's ops for one config-3 decode token on the host cores, the way
    TurboEngineV7MoE.forward composes them (turbo_engine_v7_moe.py:1540-2120): per layer
    quant_matmul_omp for q / k / v / o, the F32 router (f32_matmul_omp) and moe_forward_omp
    over the 8 selected experts; the output head is the reference's Q8_0 requantization of
    the Q6_K head (turbo_engine_v7_moe.py:515-518) through quant_matmul_omp.  One layer is
    timed and counted 48 times (the layers are the same work); attention over a 128-token
    context and the norms are left out (small next to the weight streaming)."""
    try:
        from oracle import ref as R
        if not R.available():
            return {"value": None, "unit": "tok/s", "cores": 0, "kind": "reference", "sample": "oracle/_ref not built"}
        eng = R.RefEngine()
        threads = os.cpu_count() or 1
        eng.set_num_threads(threads)
        c = Q3
        N, inner, kv, E, M, V = c["N"], c["NH"] * c["HD"], c["NKH"] * c["HD"], c["E"], c["M"], c["V"]
        src = b.bc

        def host(ptr, nbytes):
            t = next(k for k in keep if k.data_ptr() <= ptr < k.data_ptr() + k.numel() * k.element_size())
            off = ptr - t.data_ptr()
            return t.view(-1).view(torch.uint8)[off:off + nbytes].cpu().numpy().copy()

        wq, wk = host(src.wQ[0], _kq_bytes(12, inner, N)), host(src.wK[0], _kq_bytes(12, kv, N))
        wv, wo = host(src.wV[0], _kq_bytes(14, kv, N)), host(src.wO[0], _kq_bytes(12, N, inner))
        router = host(src.w_gate_inp[0], E * N * 4).view(np.float32)
        ge = host(src.w_gate_exps[0], _kq_bytes(12, E * M, N))
        ue = host(src.w_up_exps[0], _kq_bytes(12, E * M, N))
        de = host(src.w_down_exps[0], _kq_bytes(14, E * N, M))
        head = np.ascontiguousarray(np.tile(host(src.wOut, _kq_bytes(8, 4096, N)), V // 4096 + 1)[: _kq_bytes(8, V, N)])
        x = np.random.default_rng(0).standard_normal(N).astype(np.float32)
        xa = np.random.default_rng(1).standard_normal(inner).astype(np.float32)
        q, k_, v_, o = (np.zeros(n, np.float32) for n in (inner, kv, kv, N))
        lg, comb = np.zeros(E, np.float32), np.zeros(N, np.float32)
        logits = np.zeros(V, np.float32)
        sel = np.arange(0, E, E // c["k"], dtype=np.int32)[: c["k"]]
        wts = np.full(c["k"], 1.0 / c["k"], np.float32)
        cu = ctypes.POINTER(ctypes.c_uint8)
        gs, us, ds = _kq_bytes(12, M, N), _kq_bytes(12, M, N), _kq_bytes(14, N, M)
        gp = (cu * E)(*[ctypes.cast(ge.ctypes.data + e * gs, cu) for e in range(E)])
        up = (cu * E)(*[ctypes.cast(ue.ctypes.data + e * us, cu) for e in range(E)])
        dp = (cu * E)(*[ctypes.cast(de.ctypes.data + e * ds, cu) for e in range(E)])
        pre = np.zeros(3 * c["k"] * M, np.float32)   # moe_forward_omp's 3 x top_k x n_ff scratch
        pre_q8 = np.zeros(M // 32 * 34 + N // 32 * 34, np.uint8)

        def layer():
            eng.so.quant_matmul_omp(R.uptr(wq), R.fptr(x), R.fptr(q), inner, N, 12)
            eng.so.quant_matmul_omp(R.uptr(wk), R.fptr(x), R.fptr(k_), kv, N, 12)
            eng.so.quant_matmul_omp(R.uptr(wv), R.fptr(x), R.fptr(v_), kv, N, 14)
            eng.so.quant_matmul_omp(R.uptr(wo), R.fptr(xa), R.fptr(o), N, inner, 12)
            eng.so.f32_matmul_omp(R.fptr(router), R.fptr(x), R.fptr(lg), E, N)
            eng.so.moe_forward_omp(gp, up, dp, R.fptr(x), M, N, 12, 12, 14, sel.ctypes.data_as(ctypes.POINTER(ctypes.c_int)),
                                   R.fptr(wts), c["k"], R.fptr(comb), R.fptr(pre), R.uptr(pre_q8))

        layer()
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds / 2 or n < 3:
            layer()
            n += 1
        t_layer = (time.perf_counter() - t0) / n
        eng.so.quant_matmul_omp(R.uptr(head), R.fptr(x), R.fptr(logits), V, N, 8)
        m, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds / 4 or m < 2:
            eng.so.quant_matmul_omp(R.uptr(head), R.fptr(x), R.fptr(logits), V, N, 8)
            m += 1
        t_head = (time.perf_counter() - t0) / m
        t_tok = c["L"] * t_layer + t_head
        return {"value": round(1.0 / t_tok, 2), "unit": "tok/s", "cores": threads, "kind": "reference",
                "sample": f"{n} timings of one layer's reference C ops (4 quant_matmul_omp, f32_matmul_omp router, "
                          f"moe_forward_omp over 8 experts) x 48 + {m} timings of the Q8_0 head, B=1",
                "ms_per_layer": round(t_layer * 1e3, 3), "ms_head": round(t_head * 1e3, 3)}
    except Exception as e:
        return {"value": None, "unit": "tok/s", "cores": 0, "kind": "reference", "sample": f"failed: {e}"}


def run_qwen3moe_profile(args):
    """Small case for an ncu launch list of config-3 decode steps: `--profile-steps` layers,
    a 4-token prompt, then 2 decode steps at B = 1 and 2 at B = 16 (weights ~1.9 GB)."""
    import torch
    from mojollama_b200 import core
    from mojollama_b200.serving import PagedKV
    lib = core()
    assert lib.mlq_init(0) == 0
    stream = torch.cuda.Stream()
    lib.mlq_set_stream(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    b, keep = build_qwen3moe(torch, lib, layers=args.profile_steps)
    lib.mlq_set_stream(ctypes.c_void_p(stream.cuda_stream))
    V = Q3["V"]
    for B in (1, 16):
        kvs = [PagedKV(args.profile_steps, Q3["NKH"], Q3["HD"], 64, 2) for _ in range(B)]
        b.kv_array([k.block for k in kvs])
        d_logits = torch.empty(B * V, device="cuda")
        b.bc.logits = ctypes.cast(ctypes.c_void_p(d_logits.data_ptr()), ctypes.POINTER(ctypes.c_float))
        d_tok = torch.zeros(B, dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            for t in range(6):
                rc = lib.mlq_batch_forward_sample(ctypes.byref(b.bc), ctypes.c_void_p(d_tok.data_ptr()), B, None,
                                                  ctypes.c_float(0.0), 0, t, ctypes.c_void_p(d_tok.data_ptr()))
                assert rc == 0, lib.mlq_last_error_message()
        stream.synchronize()
        for k in kvs:
            k.free()
    print(json.dumps({"qwen3moe_profile_layers": args.profile_steps}))
    return 0


def run_qwen3moe_only(args):
    import torch
    from mojollama_b200 import core
    lib = core()
    assert lib.mlq_init(0) == 0
    stream = torch.cuda.Stream()
    lib.mlq_set_stream(ctypes.c_void_p(stream.cuda_stream))
    print(json.dumps({"qwen3moe": run_qwen3moe(torch, lib, stream, with_cpu=not args.no_cpu_baseline,
                                               cpu_seconds=args.cpu_seconds)}), flush=True)
    return 0


# ------------------------------------------------------------------------------ config-4 whole model
# GPT-OSS-20B shape through batch_forward: 24 layers, d_model 2880, 64 / 8 heads of 64, bf16
# attention projections, layers alternating full and 128-token sliding-window attention
# (mlq_set_attention_windows), 32 MXFP4 experts top-4 with SwiGLU FFN 2880, F32 router, bf16
# head over 201088 tokens, KV in 16-token pages.  Decode 128 steps after a 1024-token
# context at B = 1, 16 and 64.  The context's K/V rows are not computed (no prefill is
# timed): the pages are mapped zero-filled, which leaves the decode step's work -- weights
# and K/V rows read -- what it is at that context.  The batch engine's MoE rule (moe_ffn: no
# renormalisation, exact SiLU) and no attention sinks.
Q4 = dict(L=24, N=2880, NH=64, NKH=8, HD=64, V=201088, E=32, k=4, M=2880, eps=1e-5, ctx=1024, gen=128, window=128)


def gptoss_step_bytes(B, pos):
    c = Q4
    N, inner, kv, M = c["N"], c["NH"] * c["HD"], c["NKH"] * c["HD"], c["M"]
    attn = 2 * (inner * N + 2 * kv * N + N * inner)
    expert = 3 * M * N // 32 * 17
    distinct = c["E"] * (1 - (1 - c["k"] / c["E"]) ** B)
    n_full = c["L"] // 2
    kv_rows = n_full * (pos + 1) + (c["L"] - n_full) * min(pos + 1, c["window"])
    kv_bytes = B * kv_rows * 2 * kv * 4 + B * c["L"] * 2 * kv * 4
    return int(c["L"] * (attn + c["E"] * N * 4 + distinct * expert) + 2 * c["V"] * N + kv_bytes +
               B * (N * 4 + c["V"] * 4)), distinct


def build_gptoss(torch, lib, layers=None):
    from mojollama_b200 import bc as BCm
    c = Q4
    L, N, NH, NKH, HD, V, E, M = layers or c["L"], c["N"], c["NH"], c["NKH"], c["HD"], c["V"], c["E"], c["M"]
    inner, kv = NH * HD, NKH * HD
    g = torch.Generator(device="cuda").manual_seed(4)
    keep = []

    def bf16(rows, cols):
        t = (torch.randn(rows * cols, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
        keep.append(t)
        return t.data_ptr()

    def mx(rows, cols):
        t = _random_blocks(torch, 39, rows * cols // 32, g)
        keep.append(t)
        return t.data_ptr()

    b = BCm.BCBuilder()
    bc = b.bc
    bc.L, bc.N, bc.NH, bc.NKH, bc.HD, bc.FF, bc.V, bc.eps, bc.nc = L, N, NH, NKH, HD, 0, V, c["eps"], N
    for nm, r, k in (("wQ", inner, N), ("wK", kv, N), ("wV", kv, N), ("wO", N, inner)):
        b.layers(nm, [bf16(r, k) for _ in range(L)])
    for f, v in (("nQ", inner), ("nK", kv), ("nV", kv), ("nO", N)):
        b.ints(f, [v] * L)
    for f in ("q_quant", "k_quant", "v_quant", "o_quant"):
        b.ints(f, [30] * L)
    ones = torch.ones(N, device="cuda")
    keep.append(ones)
    b.layers("wAN", [ones.data_ptr()] * L)
    b.layers("wFN", [ones.data_ptr()] * L)
    routers = [torch.randn(E * N, generator=g, device="cuda") * (1.0 / np.sqrt(N)) for _ in range(L)]
    keep.extend(routers)
    b.layers("w_gate_inp", [r.data_ptr() for r in routers])
    b.layers("w_gate_exps", [mx(E * M, N) for _ in range(L)])
    b.layers("w_up_exps", [mx(E * M, N) for _ in range(L)])
    b.layers("w_down_exps", [mx(E * N, M) for _ in range(L)])
    bc.n_experts, bc.n_experts_per_tok, bc.moe_intermediate = E, c["k"], M
    bc.gate_exp_quant, bc.up_exp_quant, bc.down_exp_quant = 39, 39, 39
    emb = torch.randn(V * N, generator=g, device="cuda") * 0.02
    keep.append(emb)
    bc.emb, bc.emb_quant = emb.data_ptr(), 0
    bc.onw = ones.data_ptr()
    bc.wOut = bf16(V, N)
    bc.outNR, bc.outNC, bc.outQuant = V, N, 30
    max_ctx = c["ctx"] + c["gen"] + 8
    j = np.arange(HD // 2)
    theta = np.arange(max_ctx)[:, None] / np.power(150000.0, 2.0 * j / HD)
    b.ptr("cos_table", np.cos(theta).astype(np.float32))
    b.ptr("sin_table", np.sin(theta).astype(np.float32))
    bc.max_ctx, bc.rope_dim = max_ctx, HD
    win = np.array([0 if l % 2 == 0 else c["window"] for l in range(L)], np.int32)
    assert lib.mlq_set_attention_windows(ctypes.byref(bc), win.ctypes.data, L) == 0
    torch.cuda.synchronize()
    return b, keep


def run_gptoss(torch, lib, stream):
    """Config 4 decode through batch_forward with device sampling, per batch size."""
    from mojollama_b200.serving import PagedKV
    c = Q4
    V, P, G = c["V"], c["ctx"], c["gen"]
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    hbm = peaks.get("hbm_gbs", 6650.0)
    prev = lib.mlq_get_stream()
    lib.mlq_set_stream(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    b, keep = build_gptoss(torch, lib)
    lib.mlq_set_stream(ctypes.c_void_p(prev))
    out = {"workload": "GPT-OSS-20B shape: 24 layers, bf16 attention alternating full / 128-token window, 32 MXFP4 "
                       "experts top-4, bf16 head over 201088 tokens, 16-token KV pages; 128 greedy decode steps after "
                       "a 1024-token context (config 4)", "context_kv": "zero-filled pages (prefill not timed)",
           "batches": {}}
    for B in (1, 16, 64):
        kvs = [PagedKV(c["L"], c["NKH"], c["HD"], 16, (P + G) // 16 + 2) for _ in range(B)]
        for k in kvs:
            k.fast_forward(P)
        b.kv_array([k.block for k in kvs])
        d_logits = torch.empty(B * V, device="cuda")
        b.bc.logits = ctypes.cast(ctypes.c_void_p(d_logits.data_ptr()), ctypes.POINTER(ctypes.c_float))
        d_tok = torch.from_numpy(np.random.default_rng(B).integers(0, V, B).astype(np.int32)).cuda()
        torch.cuda.synchronize()

        def fwd(t):
            rc = lib.mlq_batch_forward_sample(ctypes.byref(b.bc), ctypes.c_void_p(d_tok.data_ptr()), B, None,
                                              ctypes.c_float(0.0), 0, t, ctypes.c_void_p(d_tok.data_ptr()))
            if rc:
                raise RuntimeError(lib.mlq_last_error_message())

        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        with torch.cuda.stream(stream):
            for t in range(3):          # warm-up (plan, first eager step, graph capture)
                fwd(t)
            ev[0].record(stream)
            l0 = lib.mlq_launch_count()
            for t in range(3, G):
                fwd(t)
            ev[1].record(stream)
        stream.synchronize()
        steps = G - 3
        launches = (lib.mlq_launch_count() - l0) // steps
        ms = ev[0].elapsed_time(ev[1]) / steps
        sb = [gptoss_step_bytes(B, P + t) for t in range(3, G)]
        step_bytes = sum(x[0] for x in sb) / steps
        achieved = step_bytes / (ms / 1e3) / 1e9
        out["batches"][str(B)] = {
            "tok_s": round(B / (ms / 1e3), 1), "ms_per_step": round(ms, 3), "launches_per_step": int(launches),
            "roofline": {"bound": "hbm", "bytes_per_step": int(step_bytes),
                         "expected_distinct_experts_per_layer": round(sb[0][1], 1),
                         "achieved_gbs": round(achieved, 1), "peak": hbm, "frac": round(achieved / hbm, 4)}}
        for k in kvs:
            k.free()
        del d_logits
    lib.mlq_set_attention_windows(ctypes.byref(b.bc), None, 0)
    del keep
    torch.cuda.empty_cache()
    return out


def run_gptoss_profile(args):
    """Small case for an ncu launch list of config-4 decode steps: `--profile-steps` layers,
    a 256-token context, 4 steps at B = 16 and 4 at B = 64 (weights ~2.7 GB)."""
    import torch
    from mojollama_b200 import core
    from mojollama_b200.serving import PagedKV
    lib = core()
    assert lib.mlq_init(0) == 0
    stream = torch.cuda.Stream()
    lib.mlq_set_stream(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    L = args.profile_steps
    b, keep = build_gptoss(torch, lib, layers=L)
    lib.mlq_set_stream(ctypes.c_void_p(stream.cuda_stream))
    V = Q4["V"]
    for B in (16, 64):
        kvs = [PagedKV(L, Q4["NKH"], Q4["HD"], 16, 24) for _ in range(B)]
        for k in kvs:
            k.fast_forward(256)
        b.kv_array([k.block for k in kvs])
        d_logits = torch.empty(B * V, device="cuda")
        b.bc.logits = ctypes.cast(ctypes.c_void_p(d_logits.data_ptr()), ctypes.POINTER(ctypes.c_float))
        d_tok = torch.zeros(B, dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            for t in range(4):
                rc = lib.mlq_batch_forward_sample(ctypes.byref(b.bc), ctypes.c_void_p(d_tok.data_ptr()), B, None,
                                                  ctypes.c_float(0.0), 0, t, ctypes.c_void_p(d_tok.data_ptr()))
                assert rc == 0, lib.mlq_last_error_message()
        stream.synchronize()
        for k in kvs:
            k.free()
    print(json.dumps({"gptoss_profile_layers": L}))
    return 0


def run_gptoss_only(args):
    import torch
    from mojollama_b200 import core
    lib = core()
    assert lib.mlq_init(0) == 0
    stream = torch.cuda.Stream()
    lib.mlq_set_stream(ctypes.c_void_p(stream.cuda_stream))
    print(json.dumps({"gptoss": run_gptoss(torch, lib, stream)}), flush=True)
    return 0


# ------------------------------------------------------------------------------ config-5 whole model
# Hybrid attention/SSM MoE (Qwen3.6-35B style) through the reference-named 76-argument
# qwen36_batch_forward (cengine_batch_instr.c:859-1231) of cengine_batch_instr.so: 40 layers
# in a repeating [3 SSM + 1 GQA] pattern, d_model 2048; GQA 16 / 2 heads of 256 with a fused
# QKV projection; SSM layers as that entry point defines them (its own ssm_decode_step,
# groups 32, state 128, inner 2048, conv 4); every layer an MoE of 256 MXFP4 experts (FF
# 512) top-8 renormalised plus a shared expert; vocab 151936.  B = 10 sequences, 128 prompt
# steps then 64 decode steps.  Attention / SSM projections and the head in Q8_0.  Synthetic
# weights: random blocks with small scales.  The entry point's own semantics (one shared
# KV slot per layer and step, cengine_batch_instr.c:1069-1072) are kept; the work per step
# -- the weights streamed -- is that of the model.  N > 1: independent replicas per GPU.
Q5 = dict(L=40, N=2048, NH=16, NKH=2, HD=256, V=151936, E=256, k=8, M=512, SI=512, IN=2048, G=32, S=128, DR=32,
          eps=1e-6, B=10, prompt=128, gen=64)
QWEN36_ARGTYPES = ([ctypes.c_int] * 10 + [ctypes.c_float] + [ctypes.c_int] * 7 + [ctypes.c_void_p, ctypes.c_int] +
                   [ctypes.c_void_p] * 39 + [ctypes.c_int] * 3 + [ctypes.c_void_p] * 14)


def _random_blocks(torch, qt, n_blocks, gen):
    """random Q8_0 / MXFP4 blocks on the device with small scales: Q8_0 d = 2^-12 (values
    up to 0.031), MXFP4 e = 119 (values up to 6 * 2^-8)"""
    bb = {8: 34, 39: 17}[qt]
    w = torch.randint(0, 256, (n_blocks, bb), dtype=torch.uint8, device="cuda", generator=gen)
    if qt == 8:
        w[:, 0], w[:, 1] = 0x00, 0x0C
    else:
        w[:, 0] = 119
    return w.reshape(-1)


def hybrid_step_bytes(B):
    c = Q5
    N, inner, n_kv, IN = c["N"], c["NH"] * c["HD"], c["NKH"] * c["HD"], c["IN"]
    q8 = lambda r, k: r * k // 32 * 34
    mx = lambda r, k: r * k // 32 * 17
    attn = q8(inner + 2 * n_kv, N) + q8(N, inner)
    ssm = q8(IN, N) + q8(N, IN)
    expert = 2 * mx(c["M"], N) + mx(N, c["M"])
    distinct = c["E"] * (1 - (1 - c["k"] / c["E"]) ** B)
    moe = c["E"] * N * 4 + expert * (distinct + 1) + N * 4
    n_attn = c["L"] // 4
    return int(n_attn * attn + (c["L"] - n_attn) * ssm + c["L"] * moe + q8(c["V"], N)), distinct


def build_hybrid(torch, L):
    c = Q5
    N, inner, n_kv, IN, E, M, SI, V = c["N"], c["NH"] * c["HD"], c["NKH"] * c["HD"], c["IN"], c["E"], c["M"], c["SI"], c["V"]
    g = torch.Generator(device="cuda").manual_seed(5)
    keep = []

    def blk(qt, rows, cols):
        t = _random_blocks(torch, qt, rows * cols // 32, g)
        keep.append(t)
        return t.data_ptr()

    def dev(t):
        keep.append(t)
        return t.data_ptr()

    types = [1 if l % 4 != 3 else 0 for l in range(L)]
    m = {"types": types, "keep": keep}
    m["an"] = [dev(torch.ones(N, device="cuda")) for _ in range(L)]
    m["fn"] = [dev(torch.ones(N, device="cuda")) for _ in range(L)]
    m["qkv"] = [blk(8, inner + 2 * n_kv, N) if t == 0 else None for t in types]
    m["o"] = [blk(8, N, inner) if t == 0 else None for t in types]
    m["gate"] = [blk(8, IN, N) if t == 1 else None for t in types]
    m["sout"] = [blk(8, N, IN) if t == 1 else None for t in types]
    m["gexp"] = [blk(39, E * M, N) for _ in range(L)]
    m["uexp"] = [blk(39, E * M, N) for _ in range(L)]
    m["dexp"] = [blk(39, E * N, M) for _ in range(L)]
    m["shg"] = [blk(39, SI, N) for _ in range(L)]
    m["shu"] = [blk(39, SI, N) for _ in range(L)]
    m["shd"] = [blk(39, N, SI) for _ in range(L)]
    m["shr"] = [dev(torch.randn(N, generator=g, device="cuda") * (1.0 / np.sqrt(N))) for _ in range(L)]
    m["router"] = [dev(torch.randn(E * N, generator=g, device="cuda") * (1.0 / np.sqrt(N))) for _ in range(L)]
    G, DR = c["G"], c["DR"]
    m["conv"] = [dev(torch.randn(2 * IN, generator=g, device="cuda") * 0.5) if t == 1 else None for t in types]
    m["sa"] = [dev(-0.5 * torch.rand(G, generator=g, device="cuda")) if t == 1 else None for t in types]
    m["sdt"] = [dev(0.1 * torch.randn(G, generator=g, device="cuda")) if t == 1 else None for t in types]
    m["sal"] = [dev(0.1 * torch.randn(G * DR, generator=g, device="cuda")) if t == 1 else None for t in types]
    m["sbe"] = [dev(0.1 * torch.randn(G * DR, generator=g, device="cuda")) if t == 1 else None for t in types]
    m["snorm"] = [dev(torch.ones(IN, device="cuda")) if t == 1 else None for t in types]
    m["emb"] = dev(torch.randn(V * N, generator=g, device="cuda") * 0.02)
    m["onw"] = dev(torch.ones(N, device="cuda"))
    m["wout"] = blk(8, V, N)
    max_ctx = c["prompt"] + c["gen"] + 8
    j = np.arange(c["HD"] // 2)
    theta = np.arange(max_ctx)[:, None] / np.power(1e7, 2.0 * j / c["HD"])
    m["cos"] = dev(torch.from_numpy(np.cos(theta).astype(np.float32)).cuda())
    m["sin"] = dev(torch.from_numpy(np.sin(theta).astype(np.float32)).cuda())
    m["max_ctx"] = max_ctx
    m["kv_k"] = dev(torch.zeros(L * max_ctx * n_kv, device="cuda"))
    m["kv_v"] = dev(torch.zeros(L * max_ctx * n_kv, device="cuda"))
    m["ssm_state"] = dev(torch.zeros(L * G * c["S"], device="cuda"))
    torch.cuda.synchronize()
    return m


class HybridCall:
    """qwen36_batch_forward's 76 arguments for the config-5 model (host arrays of device
    pointers and sizes kept alive here)."""

    def __init__(self, m, L):
        c = Q5
        self.m, self.L, self.keep = m, L, []
        N, inner, n_kv, IN = c["N"], c["NH"] * c["HD"], c["NKH"] * c["HD"], c["IN"]

        def P(items):
            arr = (ctypes.c_void_p * L)(*items)
            self.keep.append(arr)
            return ctypes.cast(arr, ctypes.c_void_p).value

        def I(vals):
            arr = np.ascontiguousarray(vals, dtype=np.int32)
            self.keep.append(arr)
            return arr.ctypes.data

        t = m["types"]
        self.kv_lens = np.zeros(L, np.int32)
        self.f = [P(m["an"]), P(m["fn"]),
                  P(m["qkv"]), I([inner + 2 * n_kv] * L), I([N] * L), I([8] * L),
                  P(m["gate"]), I([IN] * L), I([N] * L), I([8] * L),
                  P(m["sout"]), I([N] * L), I([IN] * L), I([8] * L),
                  P(m["o"]), I([N] * L), I([inner] * L), I([8] * L),
                  P(m["gexp"]), I([39] * L), P(m["uexp"]), I([39] * L), P(m["dexp"]), I([39] * L),
                  P(m["shg"]), P(m["shu"]), P(m["shd"]), P(m["shr"]), I([c["SI"]] * L),
                  P(m["router"]), I([0] * L), I([39] * L), I([39] * L), I([39] * L)]
        self.tail = [P(m["conv"]), P(m["sa"]), P(m["sdt"]), P(m["sal"]), P(m["sbe"]), P(m["snorm"])]
        self.types = I(t)

    def __call__(self, fn, tokens_ptr, B, logits_ptr, ws_ptr):
        c, m = Q5, self.m
        fn.argtypes = QWEN36_ARGTYPES
        fn.restype = None
        fn(B, self.L, c["N"], c["NH"], c["NKH"], c["HD"], 0, c["E"], c["k"], c["M"], c["eps"], c["HD"],
           m["max_ctx"], c["IN"], c["G"], c["S"], 4, c["DR"], m["emb"], 0, self.types, tokens_ptr, logits_ptr,
           *self.f, m["onw"], m["wout"], c["V"], c["N"], 8, *self.tail, m["ssm_state"], m["kv_k"], m["kv_v"],
           self.kv_lens.ctypes.data, m["cos"], m["sin"], ws_ptr, None)


def run_hybrid(torch, lib, stream, rank=0, world=1):
    """Config 5: B = 10 sequences through qwen36_batch_forward with device weights, tokens
    and logits (the drop-in's asynchronous form: every pointer is device memory), greedy
    next tokens on the device (mlq_argmax); timed over the 64 decode steps after a 128-step
    prompt.  Returns this rank's numbers (the caller takes the max over ranks)."""
    from mojollama_b200.kernels import load_kernels
    c = Q5
    B, V, P, G = c["B"], c["V"], c["prompt"], c["gen"]
    prev = lib.mlq_get_stream()
    lib.mlq_set_stream(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    m = build_hybrid(torch, c["L"])
    lib.mlq_set_stream(ctypes.c_void_p(prev))
    call = HybridCall(m, c["L"])
    fn = load_kernels().cengine.qwen36_batch_forward
    d_logits = torch.empty(B * V, device="cuda")
    d_tok = torch.zeros(B, dtype=torch.int32, device="cuda")
    prompts = torch.from_numpy(np.random.default_rng(7 + rank).integers(0, V, (P, B)).astype(np.int32)).cuda()
    ws = torch.empty(12 * B * 8192 + 8, device="cuda")
    torch.cuda.synchronize()

    def step(t):
        call(fn, d_tok.data_ptr(), B, d_logits.data_ptr(), ws.data_ptr())
        call.kv_lens += 1            # the caller advances the per-layer cache lengths
        rc = lib.mlq_argmax(ctypes.c_void_p(d_logits.data_ptr()), B, V, ctypes.c_void_p(d_tok.data_ptr()))
        if rc or lib.mlq_last_error():
            raise RuntimeError(lib.mlq_last_error_message())

    evs = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    with torch.cuda.stream(stream):
        evs[0].record(stream)
        for t in range(P):
            d_tok.copy_(prompts[t])
            step(t)
        evs[1].record(stream)
        l0 = lib.mlq_launch_count()
        for t in range(G):
            step(P + t)
        evs[2].record(stream)
    stream.synchronize()
    launches = (lib.mlq_launch_count() - l0) // G
    pre_ms, dec_ms = evs[0].elapsed_time(evs[1]), evs[1].elapsed_time(evs[2])
    del m, call
    torch.cuda.empty_cache()
    return {"dec_ms": dec_ms, "pre_ms": pre_ms, "launches": launches}


def run_hybrid_profile(args):
    """Small case for an ncu launch list of config-5 decode steps: `--profile-steps` layers
    ([3 SSM + 1 GQA] repeating), B = 10, 4 qwen36_batch_forward steps after 2 warm-up steps.
    Prints the host time to issue one step and the device time of that step."""
    import time

    import torch
    from mojollama_b200 import core
    from mojollama_b200.kernels import load_kernels
    lib = core()
    assert lib.mlq_init(0) == 0
    stream = torch.cuda.Stream()
    lib.mlq_set_stream(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    L = args.profile_steps
    m = build_hybrid(torch, L)
    lib.mlq_set_stream(ctypes.c_void_p(stream.cuda_stream))
    call = HybridCall(m, L)
    fn = load_kernels().cengine.qwen36_batch_forward
    B, V = Q5["B"], Q5["V"]
    d_logits = torch.empty(B * V, device="cuda")
    d_tok = torch.zeros(B, dtype=torch.int32, device="cuda")
    ws = torch.empty(12 * B * 8192 + 8, device="cuda")
    torch.cuda.synchronize()
    host_ms, dev_ms = [], []
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        for t in range(6):
            stream.synchronize()
            e0.record(stream)
            t0 = time.perf_counter()
            call(fn, d_tok.data_ptr(), B, d_logits.data_ptr(), ws.data_ptr())
            t1 = time.perf_counter()
            e1.record(stream)
            call.kv_lens += 1
            assert lib.mlq_argmax(ctypes.c_void_p(d_logits.data_ptr()), B, V, ctypes.c_void_p(d_tok.data_ptr())) == 0
            stream.synchronize()
            if t >= 2:
                host_ms.append((t1 - t0) * 1e3)
                dev_ms.append(e0.elapsed_time(e1))
    print(json.dumps({"hybrid_profile_layers": L, "host_issue_ms": [round(x, 3) for x in host_ms],
                      "device_ms": [round(x, 3) for x in dev_ms]}))
    return 0


def hybrid_line(res, world):
    c = Q5
    B, G, P = c["B"], c["gen"], c["prompt"]
    bytes_step, distinct = hybrid_step_bytes(B)
    ms = res["dec_ms"] / G
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    hbm = peaks.get("hbm_gbs", 6650.0)
    achieved = bytes_step / (ms / 1e3) / 1e9
    return {"workload": "hybrid [3 SSM + 1 GQA] x 10, 256 MXFP4 experts top-8 + shared expert, Q8_0 projections, "
                        "B=10 x (128 prompt + 64 greedy) through qwen36_batch_forward (config 5); N > 1: one "
                        "independent replica per GPU",
            "replicas": world, "tok_s": round(world * B * G / (res["dec_ms"] / 1e3), 1),
            "tok_s_per_replica": round(B * G / (res["dec_ms"] / 1e3), 1), "ms_per_step": round(ms, 3),
            "prefill_tok_s": round(world * B * P / (res["pre_ms"] / 1e3), 1), "launches_per_step": res["launches"],
            "roofline": {"bound": "hbm", "bytes_per_step": bytes_step,
                         "expected_distinct_experts_per_layer": round(distinct, 1),
                         "achieved_gbs": round(achieved, 1), "peak": hbm, "frac": round(achieved / hbm, 4)}}


def run_hybrid_only(args, rank, world, local_rank):
    import datetime

    import torch
    import torch.distributed as dist
    from mojollama_b200 import core
    torch.cuda.set_device(local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        lib = core()
        assert lib.mlq_init(local_rank) == 0
        stream = torch.cuda.Stream()
        lib.mlq_set_stream(ctypes.c_void_p(stream.cuda_stream))
        res = run_hybrid(torch, lib, stream, rank, world)
        t = torch.tensor([res["dec_ms"], res["pre_ms"]], device="cuda")
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res["dec_ms"], res["pre_ms"] = (float(v) for v in t.tolist())
        if rank == 0:
            print(json.dumps({"hybrid": hybrid_line(res, world)}), flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()
    return 0


SWEEP_SHAPES = [(2048, 2048), (5632, 2048), (2880, 2880), (151936, 2048)]
SWEEP_M = [1, 4, 16, 64, 256]


def run_sweep(args):
    """Config 2 in full as its own JSON object (see sweep_cases)."""
    import torch
    from mojollama_b200 import core
    lib = core()
    assert lib.mlq_init(0) == 0
    stream = torch.cuda.Stream()
    lib.mlq_set_stream(ctypes.c_void_p(stream.cuda_stream))
    ms = [int(v) for v in args.sweep_m.split(",")] if args.sweep_m else SWEEP_M
    print(json.dumps(sweep_cases(torch, lib, stream, ms)), flush=True)
    return 0


def sweep_cases(torch, lib, stream, ms):
    """Config 2 in full: every format x shape x M, device-resident, CUDA events,
    weights rotated over enough distinct copies that each launch reads from HBM (the set
    of copies is > 2x L2).  GB/s (algorithmic bytes) and TFLOP/s (2*M*N*K) per case."""
    from mojollama_b200 import gguf_quant as Q
    out = {"metric": "config-2 sweep: GB/s = (N*row_bytes + M*K*4 + M*N*4)/t, TFLOP/s = 2*M*N*K/t", "cases": []}
    for name, qt in FORMATS:
        be, bb = BLOCK[qt]
        for (n, k) in SWEEP_SHAPES:
            if k % be:
                continue
            rb = k // be * bb
            rng = np.random.default_rng(qt * 7 + n)
            distinct = min(n, 1024)
            base = Q.quantize(qt, (rng.standard_normal(distinct * k) * 0.02).astype(np.float32))
            w1 = np.tile(base, -(-n // distinct))[: n * rb]
            mat = n * rb
            copies = max(1, min(64, int(2 * 126e6 // mat) + 1))
            dev = torch.from_numpy(np.ascontiguousarray(np.tile(w1, copies))).cuda()
            for m in ms:
                x = torch.randn(m * k, device="cuda")
                o = torch.empty(m * n, device="cuda")
                torch.cuda.synchronize()   # x and the weights were written on torch's stream

                def launch(i):
                    rc = lib.mlq_matmul(ctypes.c_void_p(dev.data_ptr() + (i % copies) * mat), qt,
                                        ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(o.data_ptr()), n, k, m)
                    if rc:
                        raise RuntimeError(lib.mlq_last_error_message())

                for i in range(3):
                    launch(i)
                reps = max(5, min(50, int(2e9 // max(mat, 1))))
                a, b2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                for i in range(reps):
                    launch(i)
                b2.record(stream)
                stream.synchronize()
                t = a.elapsed_time(b2) / reps / 1e3
                byts = mat + m * k * 4 + m * n * 4
                out["cases"].append({"fmt": name, "N": n, "K": k, "M": m, "us": round(t * 1e6, 2),
                                     "gbs": round(byts / t / 1e9, 1), "tflops": round(2 * m * n * k / t / 1e12, 2)})
            del dev
            torch.cuda.empty_cache()
    return out


def run_moe_ep_only(args, rank, world, local_rank):
    import datetime

    import torch
    import torch.distributed as dist
    from mojollama_b200 import core
    torch.cuda.set_device(local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        lib = core()
        assert lib.mlq_init(local_rank) == 0
        lib.mlq_set_stream(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        res = run_moe_ep(torch, lib, rank, world, tokens=args.moe_tokens, steps=args.moe_steps,
                         warmup=args.moe_warmup, layers=args.moe_layers)
        if rank == 0:
            print(json.dumps({"moe_ep": res, "n_gpus": world}), flush=True)
    finally:
        if world > 1:
            dist.destroy_process_group()
    return 0


def run_decode_only(args):
    import torch
    from mojollama_b200 import core
    lib = core()
    assert lib.mlq_init(0) == 0
    stream = torch.cuda.Stream()
    lib.mlq_set_stream(ctypes.c_void_p(stream.cuda_stream))
    print(json.dumps({"decode": run_decode(torch, lib, stream, with_cpu=not args.no_cpu_baseline,
                                           cpu_seconds=args.cpu_seconds, with_parity=not args.no_parity)}),
          flush=True)
    return 0


# ------------------------------------------------------------------------------ model decode
# Config 1: TinyLlama-1.1B architecture, Q8_0 weights N(0, 0.02) from seed 0,
# norms 1.0, B = 4 sequences, 16 prompt tokens each uniform in [0, 32000) from seed 0, then
# 32 greedy tokens -- one batch_forward call per position (the batch engine's decode step).
TL = dict(L=22, N=2048, NH=32, NKH=4, HD=64, FF=5632, V=32000, eps=1e-5, B=4, prompt=16, gen=32)


def tinyllama_step_bytes(pos):
    """Algorithmic HBM bytes of one decode step at position pos (0-based) for B sequences:
    every weight once (Q8_0, 34 B per 32) + the embedding rows + K/V rows read and written."""
    c = TL
    N, FF, kv = c["N"], c["FF"], c["NKH"] * c["HD"]
    per_layer = (N * N * 2 + kv * N * 2 + FF * N * 3) // 32 * 34 + 2 * N * 4
    weights = c["L"] * per_layer + c["V"] * N // 32 * 34 + N * 4
    kv_bytes = c["B"] * c["L"] * 2 * kv * 4 * (pos + 2)
    act = c["B"] * (N * 4 + c["V"] * 4)
    return weights + kv_bytes + act


def build_tinyllama(torch, lib, max_ctx):
    """Random-init TinyLlama-shape model in HBM (Q8_0 by this library's quantizer) behind a
    BC; returns (builder, device tensors, host copies for the reference, kv caches)."""
    from mojollama_b200 import bc as BCm
    c = TL
    L, N, NH, NKH, HD, FF, V = c["L"], c["N"], c["NH"], c["NKH"], c["HD"], c["FF"], c["V"]
    g = torch.Generator(device="cuda").manual_seed(0)
    keep = []

    def q8(rows, cols):
        w = torch.randn(rows * cols, generator=g, device="cuda") * 0.02
        q = torch.empty(rows * cols // 32 * 34, dtype=torch.uint8, device="cuda")
        rc = lib.mlq_quantize_q8_0(ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(q.data_ptr()), rows * cols)
        assert rc == 0, lib.mlq_last_error_message()
        keep.append(q)
        return q.data_ptr()

    # the library quantizes on torch's current stream while the model is built, so that each
    # quantize kernel follows the torch.randn that fills its input and the temporary input
    # is not reused by the caching allocator before the kernel has read it
    prev_stream = lib.mlq_get_stream()
    assert lib.mlq_set_stream(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
    b = BCm.BCBuilder()
    bc = b.bc
    bc.L, bc.N, bc.NH, bc.NKH, bc.HD, bc.FF, bc.V, bc.eps, bc.nc = L, N, NH, NKH, HD, FF, V, c["eps"], N
    names = [("wQ", N, N), ("wK", NKH * HD, N), ("wV", NKH * HD, N), ("wO", N, N), ("wG", FF, N), ("wU", FF, N),
             ("wD", N, FF)]
    ptrs = {nm: [] for nm, _, _ in names}
    for l in range(L):
        for nm, r, k in names:
            ptrs[nm].append(q8(r, k))
    for nm, r, k in names:
        b.layers(nm, ptrs[nm])
    for f, v in (("nQ", N), ("nK", NKH * HD), ("nV", NKH * HD), ("nO", N), ("nG", FF), ("nU", FF), ("nD", N)):
        b.ints(f, [v] * L)
    for f in ("q_quant", "k_quant", "v_quant", "o_quant", "g_quant", "u_quant", "d_quant"):
        b.ints(f, [8] * L)
    ones = torch.ones(N, device="cuda")
    keep.append(ones)
    b.layers("wAN", [ones.data_ptr()] * L)
    b.layers("wFN", [ones.data_ptr()] * L)
    emb = torch.randn(V * N, generator=g, device="cuda") * 0.02
    keep.append(emb)
    bc.emb = emb.data_ptr()
    bc.onw = ones.data_ptr()
    bc.wOut = q8(V, N)
    bc.outNR, bc.outNC, bc.outQuant, bc.emb_quant = V, N, 8, 0
    hd2 = HD // 2
    j = np.arange(hd2)
    theta = np.arange(max_ctx)[:, None] / np.power(10000.0, 2.0 * j / HD)
    cos_t, sin_t = np.cos(theta).astype(np.float32), np.sin(theta).astype(np.float32)
    b.ptr("cos_table", cos_t)
    b.ptr("sin_table", sin_t)
    bc.max_ctx, bc.rope_dim = max_ctx, HD
    caches = [BCm.KVCache(L, NKH, HD) for _ in range(c["B"])]
    b.kv_array([kv.block for kv in caches])
    torch.cuda.synchronize()
    assert lib.mlq_set_stream(ctypes.c_void_p(prev_stream)) == 0
    return b, keep, caches


def tinyllama_oracle_model(keep, b):
    """The oracle's model description (oracle/model.py) of the bench's TinyLlama-shape
    model: host copies of the same device bytes the library computes with."""
    c = TL
    L, N, NH, NKH, HD, FF, V = c["L"], c["N"], c["NH"], c["NKH"], c["HD"], c["FF"], c["V"]
    import torch
    src = b.bc

    def host(ptr, nbytes, dtype=np.uint8):
        t = next(k for k in keep if k.data_ptr() <= ptr < k.data_ptr() + k.numel() * k.element_size())
        off = ptr - t.data_ptr()
        return t.view(-1).view(torch.uint8)[off:off + nbytes].cpu().numpy().view(dtype).copy()

    kv = NKH * HD
    shapes = {"q": ("wQ", N, N), "k": ("wK", kv, N), "v": ("wV", kv, N), "o": ("wO", N, N), "gate": ("wG", FF, N),
              "up": ("wU", FF, N), "down": ("wD", N, FF)}
    layers = []
    for l in range(L):
        ly = {"type": "attn", "an": host(src.wAN[l], N * 4, np.float32), "fn": host(src.wFN[l], N * 4, np.float32)}
        for key, (fld, r, k) in shapes.items():
            ly[key] = (host(getattr(src, fld)[l], r * k // 32 * 34), 8)
        layers.append(ly)
    from oracle import ops as O
    cos_t, sin_t = O.rope_tables(src.max_ctx, HD, HD)
    return dict(L=L, N=N, NH=NH, NKH=NKH, HD=HD, FF=FF, V=V, eps=c["eps"], rope_dim=HD, max_ctx=src.max_ctx,
                emb=host(src.emb, V * N * 4, np.float32).reshape(V, N), onw=host(src.onw, N * 4, np.float32),
                wout=(host(src.wOut, V * N // 32 * 34), 8), cos=cos_t, sin=sin_t, moe=None, layers=layers)


def decode_parity(keep, b, fed, logits, tol=3e-3, margin=1e-2):
    """Config-1 parity at full size: the oracle (oracle/model.py forward_sequence, float64
    accumulation over the exactly decoded Q8_0 weights) fed the tokens the library was fed
    (prompts, then its own greedy tokens), position by position.  Reports the relative L2
    of every position's logits (bar: 3e-3, three layers of 1e-3-bounded ops) and the
    greedy tokens: where the oracle's top-2 margin exceeds 1e-2 the argmax must agree."""
    try:
        from oracle import model as OM
        from oracle import ops as O
        t0 = time.perf_counter()
        m = tinyllama_oracle_model(keep, b)
        want = OM.forward_sequence(m, fed)
        P, B, V = logits.shape
        rel = [O.rel_l2(logits[p], want[p]) for p in range(P)]
        top2 = np.sort(want, axis=-1)[..., -2:]
        decided = (top2[..., 1] - top2[..., 0]) > margin
        agree = np.argmax(logits, -1) == np.argmax(want, -1)
        return {"oracle": "oracle/model.py forward_sequence (numpy, float64 accumulation; pinned to the "
                          "reference C build on small models)",
                "positions": int(P), "sequences": int(B),
                "logits_rel_l2_vs_oracle": float(max(rel)), "logits_rel_l2_median": float(np.median(rel)),
                "tolerance": tol, "greedy_margin": margin,
                "greedy_decided": int(decided.sum()), "greedy_agree_where_decided": int((agree & decided).sum()),
                "greedy_agree_all": int(agree.sum()),
                "ok": bool(max(rel) <= tol and bool(np.all(agree[decided]))),
                "rel_l2_per_position": [float(f"{r:.3g}") for r in rel],
                "oracle_seconds": round(time.perf_counter() - t0, 1)}
    except Exception as e:  # never let the checker break the bench line
        return {"ok": False, "failed": f"{type(e).__name__}: {e}"}


def run_decode(torch, lib, stream, with_cpu=True, cpu_seconds=10.0, with_parity=True):
    """Config 1 through batch_forward: device-resident (logits and tokens in HBM, greedy
    argmax on the device) and end to end (host tokens and logits, the reference's usage)."""
    c = TL
    B, V, N, P, G = c["B"], c["V"], c["N"], c["prompt"], c["gen"]
    max_ctx = 64
    b, keep, caches = build_tinyllama(torch, lib, max_ctx)
    rng = np.random.default_rng(0)
    prompts = rng.integers(0, V, (B, P)).astype(np.int32)
    d_logits = torch.empty(B * V, device="cuda")
    d_tok = torch.empty(B, dtype=torch.int32, device="cuda")
    d_prompts = torch.from_numpy(np.ascontiguousarray(prompts.T)).cuda()
    bc = b.bc

    def reset():
        for kv in caches:
            lib.mlq_kv_free(ctypes.byref(kv.block))
            assert lib.mlq_kv_init(ctypes.byref(kv.block), c["L"], c["NKH"], c["HD"]) == 0
        b.kv_array([kv.block for kv in caches])

    def fwd():
        rc = lib.mlq_batch_forward(ctypes.byref(bc), ctypes.c_void_p(d_tok.data_ptr()), B, None)
        if rc:
            raise RuntimeError(lib.mlq_last_error_message())

    def generate(ev=None):
        """prompt positions then greedy positions, all on the device; ev: per-phase events"""
        bc.logits = ctypes.cast(ctypes.c_void_p(d_logits.data_ptr()), ctypes.POINTER(ctypes.c_float))
        with torch.cuda.stream(stream):
            if ev:
                ev[0].record(stream)
            for t in range(P):
                d_tok.copy_(d_prompts[t])
                fwd()
            if ev:
                ev[1].record(stream)
            for t in range(G):
                d_tok.copy_(torch.argmax(d_logits.view(B, V), dim=1).to(torch.int32))
                fwd()
            if ev:
                ev[2].record(stream)

    generate()            # warm-up (plan, residency, graphs of nothing)
    stream.synchronize()
    reset()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    l0 = lib.mlq_launch_count()
    generate(evs)
    stream.synchronize()
    launches = (lib.mlq_launch_count() - l0) // (P + G)
    pre_ms, dec_ms = evs[0].elapsed_time(evs[1]), evs[1].elapsed_time(evs[2])
    greedy_dev = torch.argmax(d_logits.view(B, V), dim=1).cpu().numpy()

    # end to end: host tokens, host logits, host argmax (the reference Python's loop)
    reset()
    h_logits = np.zeros(B * V, np.float32)
    bc.logits = h_logits.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    from mojollama_b200.kernels import load_kernels
    ce = load_kernels().cengine
    ws = np.zeros(B * N, np.float32)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for t in range(P):
        tok = np.ascontiguousarray(prompts[:, t])
        ce.batch_forward(ctypes.byref(bc), tok.ctypes.data, B, ws.ctypes.data)
    t1 = time.perf_counter()
    for t in range(G):
        tok = np.argmax(h_logits.reshape(B, V), axis=1).astype(np.int32)
        ce.batch_forward(ctypes.byref(bc), tok.ctypes.data, B, ws.ctypes.data)
    t2 = time.perf_counter()
    assert lib.mlq_last_error() == 0, lib.mlq_last_error_message()
    greedy_host = np.argmax(h_logits.reshape(B, V), axis=1)
    step_bytes = sum(tinyllama_step_bytes(P + t) for t in range(G)) / G

    parity = None
    if with_parity:
        # untimed: the same generation with every position's logits kept, then the oracle
        # fed the same tokens (teacher-forced) on host copies of the same weights
        reset()
        bc.logits = ctypes.cast(ctypes.c_void_p(d_logits.data_ptr()), ctypes.POINTER(ctypes.c_float))
        all_logits = torch.empty((P + G, B, V), device="cuda")
        fed = torch.empty((P + G, B), dtype=torch.int32, device="cuda")
        with torch.cuda.stream(stream):
            for t in range(P + G):
                if t < P:
                    d_tok.copy_(d_prompts[t])
                else:
                    d_tok.copy_(torch.argmax(all_logits[t - 1], dim=1).to(torch.int32))
                fed[t].copy_(d_tok)
                fwd()
                all_logits[t].copy_(d_logits.view(B, V))
        stream.synchronize()
        parity = decode_parity(keep, b, fed.cpu().numpy(), all_logits.cpu().numpy())
    out = {
        "workload": "TinyLlama-1.1B shape, Q8_0, B=4 x (16 prompt + 32 greedy) through batch_forward (config 1)",
        "tok_s": round(B * G / (dec_ms / 1e3), 1), "ms_per_step": round(dec_ms / G, 3),
        "prefill_tok_s": round(B * P / (pre_ms / 1e3), 1),
        "e2e_tok_s": round(B * G / (t2 - t1), 1), "e2e_ms_per_step": round((t2 - t1) * 1e3 / G, 3),
        "e2e_io": {"h2d_bytes_per_step": B * 4, "d2h_bytes_per_step": B * V * 4 + B * N * 4},
        "launches_per_step": int(launches),
        # self-consistency of the library (device argmax loop vs host argmax loop);
        # the comparison with the oracle is `parity`
        "device_and_host_loop_tokens_agree": bool(np.array_equal(greedy_dev, greedy_host)),
        "parity": parity,
        "roofline": {"bound": "hbm", "bytes_per_step": int(step_bytes),
                     "achieved_gbs": round(step_bytes / (dec_ms / G / 1e3) / 1e9, 1)},
    }
    if with_cpu:
        out["cpu_baseline"] = decode_cpu_baseline(keep, b, caches, cpu_seconds)
    for kv in caches:
        kv.free()
    return out


def decode_cpu_baseline(keep, b, caches, seconds):
    """The reference C batch_forward (oracle/_ref) on the host cores with host copies of
    the same weights, B = 4, one token per sequence per call; a bounded number of steps."""
    try:
        from oracle import ref as R
        from mojollama_b200 import bc as BCm
        if not R.available():
            return {"value": None, "unit": "tok/s", "cores": 0, "kind": "reference", "sample": "oracle/_ref not built"}
        import torch
        eng = R.RefEngine()
        threads = os.cpu_count() or 1
        eng.set_num_threads(threads)
        c = TL
        src = b.bc
        hb = BCm.BCBuilder()
        hc = hb.bc
        for name, _ in BCm.BC._fields_:
            setattr(hc, name, getattr(src, name))
        host = {}

        def to_host(ptr, nbytes):
            if ptr not in host:
                t = torch.empty(nbytes, dtype=torch.uint8)
                src_t = next(k for k in keep if k.data_ptr() <= ptr < k.data_ptr() + k.numel() * k.element_size())
                off = ptr - src_t.data_ptr()
                t.copy_(src_t.view(torch.uint8)[off:off + nbytes].cpu())
                host[ptr] = t
            return host[ptr].data_ptr()

        L, N, FF, V, kv = c["L"], c["N"], c["FF"], c["V"], c["NKH"] * c["HD"]
        sizes = {"wQ": N * N, "wK": kv * N, "wV": kv * N, "wO": N * N, "wG": FF * N, "wU": FF * N, "wD": N * FF}
        for nm, n in sizes.items():
            arr = getattr(src, nm)
            hb.layers(nm, [to_host(arr[l], n // 32 * 34) for l in range(L)])
        hb.layers("wAN", [to_host(src.wAN[0], N * 4)] * L)
        hb.layers("wFN", [to_host(src.wFN[0], N * 4)] * L)
        hc.emb = to_host(src.emb, V * N * 4)
        hc.onw = to_host(src.onw, N * 4)
        hc.wOut = to_host(src.wOut, V * N // 32 * 34)
        kvs = [BCm.KVBlock() for _ in range(c["B"])]
        for k in kvs:
            eng.so.kv_init(ctypes.byref(k), L, c["NKH"], c["HD"])
        hb.kv_array(kvs)
        logits = np.zeros(c["B"] * V, np.float32)
        hb.ptr("logits", logits)
        work = np.zeros(64 * kv * 2 + 4096, np.float32)
        hb.ptr("workspace", work)
        hc.ws_size = work.size
        S = max(N, c["NH"] * c["HD"], FF, 8192)
        ws = np.zeros(12 * c["B"] * S, np.float32)
        tok = np.zeros(c["B"], np.int32)
        eng.so.batch_forward(ctypes.byref(hc), tok.ctypes.data, c["B"], ws.ctypes.data)   # warm
        n, t0 = 0, time.perf_counter()
        while (time.perf_counter() - t0 < seconds or n < 2) and n < 40:
            eng.so.batch_forward(ctypes.byref(hc), tok.ctypes.data, c["B"], ws.ctypes.data)
            n += 1
        dt = (time.perf_counter() - t0) / n
        return {"value": round(c["B"] / dt, 2), "unit": "tok/s", "cores": threads, "kind": "reference",
                "sample": f"{n} batch_forward steps (B=4, positions 1..{n}) of the reference C engine"}
    except Exception as e:
        return {"value": None, "unit": "tok/s", "cores": 0, "kind": "reference", "sample": f"failed: {e}"}


def run_profile_tc(fmt: str, rows: int, m: int, launches: int = 3) -> int:
    """Small case for ncu on the tensor-core GEMM: one format, rows x 2048 weights, M tokens,
    two warm-up launches then `launches` more (weights ~143 MB for Q8_0 at 65536 rows)."""
    import torch
    from mojollama_b200 import core
    from mojollama_b200 import gguf_quant as Q
    qt = dict(FORMATS)[fmt]
    lib = core()
    assert lib.mlq_init(0) == 0
    rng = np.random.default_rng(qt)
    base = Q.quantize(qt, (rng.standard_normal(DISTINCT * K_COLS) * 0.02).astype(np.float32))
    w = np.tile(base, -(-rows // DISTINCT))[: rows * row_bytes(qt)]
    wd = torch.from_numpy(np.ascontiguousarray(w)).cuda()
    x = torch.randn(m * K_COLS, device="cuda")
    out = torch.empty(m * rows, device="cuda")
    lib.mlq_set_stream(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    for _ in range(2 + launches):
        rc = lib.mlq_matmul(ctypes.c_void_p(wd.data_ptr()), qt, ctypes.c_void_p(x.data_ptr()),
                            ctypes.c_void_p(out.data_ptr()), rows, K_COLS, m)
        assert rc == 0, lib.mlq_last_error_message()
    torch.cuda.synchronize()
    print(json.dumps({"profile_tc": fmt, "rows": rows, "cols": K_COLS, "m": m,
                      "flops_per_launch": 2 * m * rows * K_COLS,
                      "bytes_per_launch": rows * row_bytes(qt) + m * K_COLS * 4 + m * rows * 4}))
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


def run_moe_profile(shape: str, launches: int = 3) -> int:
    """Small case for ncu of the grouped MXFP4 expert kernels: `shape` = E,N,FF,R (experts,
    model width, expert width, routed rows), random MXFP4 experts with small scales, rows
    spread uniformly over the experts; mlq_moe_rows two warm-up calls then `launches` more.
    Prints each call's device time and the expert bytes it streams."""
    import torch
    from mojollama_b200 import core
    E, N, FF, R = (int(v) for v in shape.split(","))
    lib = core()
    assert lib.mlq_init(0) == 0
    lib.mlq_set_stream(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    g = torch.Generator(device="cuda").manual_seed(3)
    rb_n, rb_f = N // 32 * 17, FF // 32 * 17
    mats = [_random_blocks(torch, 39, E * FF * N // 32, g), _random_blocks(torch, 39, E * FF * N // 32, g),
            _random_blocks(torch, 39, E * N * FF // 32, g)]
    eid = torch.from_numpy(np.random.default_rng(5).integers(0, E, R).astype(np.int32)).cuda()
    x = torch.randn(R, N, device="cuda") * 0.5
    y = torch.empty(R, N, device="cuda")
    active = int(torch.unique(eid).numel())
    vp = lambda t: ctypes.c_void_p(t.data_ptr())
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    times = []
    for i in range(2 + launches):
        evs[0].record()
        rc = lib.mlq_moe_rows(39, 39, 39, vp(mats[0]), vp(mats[1]), vp(mats[2]), rb_n * FF, rb_n * FF, rb_f * N, E,
                              vp(eid), R, FF, N, vp(x), vp(y))
        evs[1].record()
        assert rc == 0, lib.mlq_last_error_message()
        torch.cuda.synchronize()
        if i >= 2:
            times.append(round(evs[0].elapsed_time(evs[1]) * 1e3, 1))
    print(json.dumps({"moe_profile": [E, N, FF, R], "active_experts": active, "us_per_call": times,
                      "expert_bytes": active * (2 * FF * rb_n + N * rb_f)}))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--profile", default=None, help="run the small single-kernel ncu case for FORMAT")
    ap.add_argument("--profile-rows", type=int, default=65536)
    ap.add_argument("--moe-profile", default=None, help="grouped MXFP4 expert case for ncu: E,N,FF,R")
    ap.add_argument("--profile-tc", default=None, help="small tensor-core GEMM case for ncu: FORMAT")
    ap.add_argument("--profile-m", type=int, default=64)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the oracle checks of the model sections")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-decode", action="store_true", help="skip the config-1 model decode section")
    ap.add_argument("--decode-only", action="store_true", help="run only the config-1 model decode section")
    ap.add_argument("--decode-profile", action="store_true", help="small decode case for an ncu launch list")
    ap.add_argument("--no-moe-ep", action="store_true", help="skip the config-3 expert-parallel MoE section")
    ap.add_argument("--moe-ep-only", action="store_true", help="run only the expert-parallel MoE section")
    ap.add_argument("--qwen3moe-only", action="store_true", help="run only the config-3 whole-model section")
    ap.add_argument("--no-qwen3moe", action="store_true", help="skip the config-3 whole-model section")
    ap.add_argument("--qwen3moe-profile", action="store_true", help="small config-3 case for an ncu launch list")
    ap.add_argument("--hybrid-only", action="store_true", help="run only the config-5 whole-model section")
    ap.add_argument("--gptoss-only", action="store_true", help="run only the config-4 whole-model section")
    ap.add_argument("--no-gptoss", action="store_true", help="skip the config-4 whole-model section")
    ap.add_argument("--gptoss-profile", action="store_true", help="small config-4 case for an ncu launch list")
    ap.add_argument("--no-hybrid", action="store_true", help="skip the config-5 whole-model section")
    ap.add_argument("--hybrid-profile", action="store_true", help="small config-5 case for an ncu launch list")
    ap.add_argument("--moe-layers", type=int, default=None)
    ap.add_argument("--moe-tokens", type=int, default=16)
    ap.add_argument("--moe-steps", type=int, default=5)
    ap.add_argument("--moe-warmup", type=int, default=3)
    ap.add_argument("--profile-steps", type=int, default=3)
    ap.add_argument("--sweep", action="store_true", help="config-2 sweep (formats x shapes x M), one JSON object")
    ap.add_argument("--sweep-m", default=None, help="comma-separated M values for --sweep")
    ap.add_argument("--no-sweep", action="store_true", help="leave the config-2 sweep out of the bench line")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.profile:
        return run_profile_case(args.profile, args.profile_rows)
    if args.profile_tc:
        return run_profile_tc(args.profile_tc, args.profile_rows, args.profile_m)
    if args.moe_profile:
        return run_moe_profile(args.moe_profile)
    if args.decode_only:
        return run_decode_only(args)
    if args.decode_profile:
        return run_decode_profile(args)
    if args.moe_ep_only:
        return run_moe_ep_only(args, rank, world, local_rank)
    if args.qwen3moe_only:
        return run_qwen3moe_only(args)
    if args.qwen3moe_profile:
        return run_qwen3moe_profile(args)
    if args.hybrid_only:
        return run_hybrid_only(args, rank, world, local_rank)
    if args.hybrid_profile:
        return run_hybrid_profile(args)
    if args.gptoss_only:
        return run_gptoss_only(args)
    if args.gptoss_profile:
        return run_gptoss_profile(args)
    if args.sweep:
        return run_sweep(args)
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
