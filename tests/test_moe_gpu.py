"""GPU parity of the MoE FFN (moe_forward_omp drop-in and the device router) against
the oracle, on the expert shapes of the baseline's MoE models, plus the reference C
engine's own output on a Q4_0 case.  Tolerance: relative L2 <= 1e-3."""
import ctypes
import os

import numpy as np
import pytest

from oracle import formats as F
from oracle import ops as O

pytestmark = pytest.mark.gpu
TOL = 1e-3
cu = ctypes.POINTER(ctypes.c_uint8)
cf = ctypes.POINTER(ctypes.c_float)
G = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def K(cuda_device):
    from mojollama_b200.kernels import load_kernels
    return load_kernels()


def experts(qt, n_exp, rows, cols, seed):
    """one 3-D expert tensor (expert-major, as GGUF stores it) + per-expert views"""
    rng = np.random.default_rng(seed)
    rb = F.row_bytes(qt, cols)
    base = F.quantize(qt, (rng.standard_normal(rows * cols) * 0.02).astype(np.float32))
    big = np.concatenate([np.roll(base, 17 * e * rb) for e in range(n_exp)])   # distinct per expert
    views = {e: big[e * rows * rb:(e + 1) * rows * rb] for e in range(n_exp)}
    return big, views


def run_moe(K, qts, n_embd, n_ff, n_exp, top_k, seed, register=False):
    qg, qu, qd = qts
    gbig, g = experts(qg, n_exp, n_ff, n_embd, seed)
    ubig, u = experts(qu, n_exp, n_ff, n_embd, seed + 1)
    dbig, d = experts(qd, n_exp, n_embd, n_ff, seed + 2)
    if register:
        from mojollama_b200 import core
        for big in (gbig, ubig, dbig):
            assert core().mlq_register_weights(big.ctypes.data, big.nbytes) == 0
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(n_embd).astype(np.float32)
    idx = rng.choice(n_exp, top_k, replace=False).astype(np.int32)
    w = rng.dirichlet(np.ones(top_k)).astype(np.float32)
    arr = cu * n_exp
    gp = arr(*[g[e].ctypes.data_as(cu) for e in range(n_exp)])
    up = arr(*[u[e].ctypes.data_as(cu) for e in range(n_exp)])
    dp = arr(*[d[e].ctypes.data_as(cu) for e in range(n_exp)])
    out = np.full(n_embd, np.nan, np.float32)
    K.kern.moe_forward_omp(gp, up, dp, x.ctypes.data_as(cf), n_ff, n_embd, qg, qu, qd,
                           idx.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), w.ctypes.data_as(cf), top_k,
                           out.ctypes.data_as(cf), None, None)
    ref = O.moe_forward(g, u, d, qts, x, n_ff, n_embd, idx, w)
    if register:
        from mojollama_b200 import core
        for big in (gbig, ubig, dbig):
            assert core().mlq_unregister_weights(big.ctypes.data) == 0
    return out, ref


@pytest.mark.parametrize("name,qts,n_embd,n_ff,n_exp,top_k", [
    ("qwen3-30b-a3b", (F.Q4_K, F.Q4_K, F.Q6_K), 2048, 768, 12, 8),
    ("gpt-oss-20b", (F.MXFP4, F.MXFP4, F.MXFP4), 2880, 2880, 5, 4),
    ("hybrid-35b", (F.MXFP4, F.MXFP4, F.MXFP4), 2048, 512, 12, 8),
    ("q8_0", (F.Q8_0, F.Q8_0, F.Q8_0), 1024, 384, 4, 2),
    ("mixed gate/up types", (F.Q4_K, F.Q5_K, F.Q8_0), 512, 256, 4, 3),
])
def test_moe_forward_omp(K, name, qts, n_embd, n_ff, n_exp, top_k):
    out, ref = run_moe(K, qts, n_embd, n_ff, n_exp, top_k, seed=n_embd + n_ff)
    assert np.all(np.isfinite(out))
    assert O.rel_l2(out, ref) < TOL, (name, O.rel_l2(out, ref))


def test_moe_forward_with_registered_expert_tensors(K):
    out, ref = run_moe(K, (F.Q4_K, F.Q4_K, F.Q6_K), 1024, 512, 8, 4, seed=5, register=True)
    assert O.rel_l2(out, ref) < TOL


def test_moe_matches_reference_c_q4_0(K):
    ro = dict(np.load(os.path.join(G, "ref_ops.npz")))
    ne, n_embd, n_ff, topk = (int(v) for v in ro["moe_dims"])
    arr = cu * ne
    mats = {k: [np.ascontiguousarray(ro[k][e]) for e in range(ne)] for k in ("moe_gate", "moe_up", "moe_down")}
    gp, up, dp = (arr(*[m.ctypes.data_as(cu) for m in mats[k]]) for k in ("moe_gate", "moe_up", "moe_down"))
    x, idx, w = ro["moe_x"], ro["moe_idx"], ro["moe_w"]
    out = np.zeros(n_embd, np.float32)
    K.kern.moe_forward_omp(gp, up, dp, x.ctypes.data_as(cf), n_ff, n_embd, 2, 2, 2,
                           idx.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), w.ctypes.data_as(cf), topk,
                           out.ctypes.data_as(cf), None, None)
    assert O.rel_l2(out, ro["moe_out"]) < TOL


@pytest.mark.parametrize("E,k,renorm", [(128, 8, 1), (32, 4, 1), (256, 8, 1), (128, 8, 0)])
def test_router(cuda_device, E, k, renorm):
    lib = cuda_device
    B, N = 5, 2048
    rng = np.random.default_rng(E + k)
    wr = (rng.standard_normal(E * N) * 0.02).astype(np.float32)
    x = rng.standard_normal(B * N).astype(np.float32)
    idx = np.zeros(B * k, np.int32)
    w = np.zeros(B * k, np.float32)
    assert lib.mlq_moe_router(x.ctypes.data, B, N, wr.ctypes.data, 0, E, k, renorm, idx.ctypes.data,
                              w.ctypes.data) == 0
    logits = O.gemv(wr.view(np.uint8), F.F32, x, E, N)
    for b in range(B):
        ei, ew = O.router_topk(logits[b], k, renorm)
        assert list(idx[b * k:(b + 1) * k]) == list(ei)
        np.testing.assert_allclose(w[b * k:(b + 1) * k], ew, rtol=1e-4, atol=1e-7)
