"""Generate the golden fixtures in tests/golden/ (run in a container that has the
reference sources and gguf-py; the fixtures themselves travel, the generators don't).

    make -C oracle                      # reference C engine from its own sources
    python tests/golden/gen_golden.py

Writes
  formats.npz  random GGUF blocks + gguf-py 0.19.0 dequantize output; gguf-py
               quantize output (Q8_0, Q4_0, MXFP4); the reference's
               quantize_row_q8_0 bytes and *_dequantize_row output.
  ref_ops.npz  outputs of the reference C engine (compiled from source, AVX2+OMP)
               on small seeded GEMV / batch-GEMV cases, including the dispatcher
               paths where the reference is not W.x (Q4_K type 12, Q6_K type 14),
               kept as evidence for the reference-compat mode.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import formats as F  # noqa: E402


def gen_formats(rng):
    import gguf
    from gguf import GGMLQuantizationType as T
    from gguf import quants
    out = {"gguf_version": np.array(gguf.__version__ if hasattr(gguf, "__version__") else "0.19.0")}
    n = 512
    for qt in (F.Q4_0, F.Q4_1, F.Q5_0, F.Q8_0, F.Q4_K, F.Q5_K, F.Q6_K, F.MXFP4, F.BF16):
        raw = F.random_blocks(qt, n, rng)
        deq = quants.dequantize(raw.reshape(1, -1), T(qt)).reshape(-1).astype(np.float32)
        out[f"deq_raw_{qt}"] = raw
        out[f"deq_out_{qt}"] = deq
    x = rng.standard_normal(256).astype(np.float32)
    out["quant_x"] = x
    for qt in (F.Q8_0, F.Q4_0, F.MXFP4):
        out[f"quant_gguf_{qt}"] = quants.quantize(x.reshape(1, -1), T(qt)).reshape(-1)
    return out


def gen_ref(rng, out):
    from oracle.ref import RefEngine
    from oracle.ref import fptr as R_fptr
    from oracle.ref import uptr as R_uptr
    ref = RefEngine()
    ref.set_num_threads(4)
    x = out["quant_x"]
    out["ref_q8_0_bytes"] = ref.quantize_row_q8_0(x)
    for qt, name in ((F.Q4_K, "q4_k"), (F.Q5_K, "q5_k"), (F.Q6_K, "q6_k"), (F.Q8_0, "q8_0")):
        out[f"ref_deq_{qt}"] = ref.dequantize_row(name, out[f"deq_raw_{qt}"], 512)
    ops = {}
    n, k = 48, 512
    for qt in (F.Q8_0, F.Q4_0, F.Q4_1, F.Q4_K, F.Q5_K, F.Q6_K, F.MXFP4_REF):
        w = F.quantize(qt, (rng.standard_normal(n * k) * 0.02).astype(np.float32))
        xv = rng.standard_normal(k).astype(np.float32)
        ops[f"gemv_w_{qt}"] = w
        ops[f"gemv_x_{qt}"] = xv
        code = 39 if qt == F.MXFP4_REF else qt
        ops[f"gemv_ref_dispatch_{qt}"] = ref.quant_matmul(w, xv, n, k, code)
    b = 3
    for qt, name in ((F.Q8_0, "q8_0"), (F.Q4_0, "q4_0"), (F.Q4_K, "q4_k"), (F.MXFP4_REF, "mxfp4")):
        w = ops[f"gemv_w_{qt}"]
        xb = rng.standard_normal(b * k).astype(np.float32)
        ops[f"bgemv_x_{qt}"] = xb
        ops[f"bgemv_ref_{qt}"] = ref.batch_matmul(name, w, xb, n, k, b)
    ops["shape"] = np.array([n, k, b], np.int32)
    # moe_forward_omp with Q4_0 experts (its gate/up/down Q4_0 paths are W.x:
    # quant_kernels_omp.c:2122-2131, 2225-2227)
    import ctypes
    ne, n_embd, n_ff, topk = 6, 256, 128, 3
    gate = [F.quantize(F.Q4_0, (rng.standard_normal(n_ff * n_embd) * 0.05).astype(np.float32)) for _ in range(ne)]
    up = [F.quantize(F.Q4_0, (rng.standard_normal(n_ff * n_embd) * 0.05).astype(np.float32)) for _ in range(ne)]
    down = [F.quantize(F.Q4_0, (rng.standard_normal(n_embd * n_ff) * 0.05).astype(np.float32)) for _ in range(ne)]
    xm = rng.standard_normal(n_embd).astype(np.float32)
    idx = np.array([4, 1, 3], np.int32)
    wt = np.array([0.5, 0.3, 0.2], np.float32)
    arr = ctypes.POINTER(ctypes.c_uint8) * ne
    gp, upp, dp = (arr(*[R_uptr(a) for a in lst]) for lst in (gate, up, down))
    comb = np.zeros(n_embd, np.float32)
    buf = np.zeros(3 * topk * n_ff, np.float32)
    q8 = np.zeros(n_embd // 32 * 34 * 4, np.uint8)
    ref.set_num_threads(1)
    ref.so.moe_forward_omp(gp, upp, dp, R_fptr(xm), n_ff, n_embd, 2, 2, 2,
                           idx.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), R_fptr(wt), topk, R_fptr(comb),
                           R_fptr(buf), R_uptr(q8))
    ops["moe_gate"], ops["moe_up"], ops["moe_down"] = np.stack(gate), np.stack(up), np.stack(down)
    ops["moe_x"], ops["moe_idx"], ops["moe_w"], ops["moe_out"] = xm, idx, wt, comb
    ops["moe_dims"] = np.array([ne, n_embd, n_ff, topk], np.int32)
    # ssm_decode_step (cengine_batch_instr.c:736), B = 3 sequences sharing one state
    B_, N_, inner_, groups_, ss_, dtr_ = 3, 64, 96, 4, 8, 5
    sx = rng.standard_normal(B_ * N_).astype(np.float32)
    sconv = rng.standard_normal(4 * 2 * inner_).astype(np.float32)
    sa = -rng.uniform(0.1, 1.0, groups_).astype(np.float32)
    sdt = rng.standard_normal(groups_).astype(np.float32)
    sal = (rng.standard_normal(groups_ * dtr_) * 0.3).astype(np.float32)
    sbe = (rng.standard_normal(groups_ * dtr_) * 0.3).astype(np.float32)
    sst = rng.standard_normal(groups_ * ss_).astype(np.float32)
    snorm = np.ones(ss_, np.float32)
    sint = np.zeros(B_ * inner_, np.float32)
    st_out = sst.copy()
    ref.so.ssm_decode_step(R_fptr(sx), R_fptr(sint), R_fptr(sconv), R_fptr(sa), R_fptr(sdt), R_fptr(sal), R_fptr(sbe),
                           R_fptr(snorm), R_fptr(st_out), B_, N_, inner_, groups_, ss_, 4, dtr_)
    for key, val in dict(ssm_x=sx, ssm_conv=sconv, ssm_a=sa, ssm_dt=sdt, ssm_alpha=sal, ssm_beta=sbe,
                         ssm_state_in=sst, ssm_interm=sint, ssm_state_out=st_out,
                         ssm_dims=np.array([B_, N_, inner_, groups_, ss_, dtr_], np.int32)).items():
        ops[key] = val
    # gqa_attention_decode (gqa_attention.c:93, built with the oracle's cblas shim).
    # Single-threaded: every OpenMP thread of the reference writes the same tmp_scores
    # buffer (gqa_attention.c:104, 113), so its multi-threaded output is a data race.
    ref.set_num_threads(1)
    if ref.gqa is not None:
        from oracle.ref import fptr
        for nh, nkh, hd, sl in ((32, 4, 64, 37), (16, 2, 256, 200)):
            qv = rng.standard_normal(nh * hd).astype(np.float32)
            kc = rng.standard_normal(sl * nkh * hd).astype(np.float32)
            vc = rng.standard_normal(sl * nkh * hd).astype(np.float32)
            out = np.zeros(nh * hd, np.float32)
            ws = np.zeros(2 * nh * sl + 16, np.float32)
            ref.gqa.gqa_attention_decode(fptr(qv), fptr(kc), fptr(vc), fptr(out), sl, nh, nkh, hd, fptr(ws))
            tag = f"{nh}_{nkh}_{hd}_{sl}"
            ops[f"gqa_q_{tag}"], ops[f"gqa_k_{tag}"], ops[f"gqa_v_{tag}"] = qv, kc, vc
            ops[f"gqa_out_{tag}"] = out
    return ops


def main():
    rng = np.random.default_rng(20261201)
    fm = gen_formats(rng)
    ops = gen_ref(rng, fm)
    np.savez_compressed(os.path.join(HERE, "formats.npz"), **fm)
    np.savez_compressed(os.path.join(HERE, "ref_ops.npz"), **ops)
    print("wrote", sorted(fm)[:4], "...", len(fm), "+", len(ops), "arrays")


if __name__ == "__main__":
    main()
