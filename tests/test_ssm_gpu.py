"""GPU parity of the reference's SSM decode step and fused SSM layer
(cengine_batch_instr.c:736-849) through cengine_batch_instr.so: the golden case from
the reference C engine, and the engine's own dimensions (groups 32, state 128,
dt_rank 32, inner 4096, N 2048, B 10; turbo_engine_v7_moe.py:228-232)."""
import ctypes
import os

import numpy as np
import pytest

from oracle import formats as F
from oracle import ops as O

pytestmark = pytest.mark.gpu
TOL = 1e-3
cf = ctypes.POINTER(ctypes.c_float)
cu = ctypes.POINTER(ctypes.c_uint8)
ci = ctypes.c_int
G = os.path.join(os.path.dirname(__file__), "golden")


def p(a):
    return a.ctypes.data_as(cf)


@pytest.fixture(scope="module")
def ce(cuda_device):
    from mojollama_b200 import load_alias
    so = load_alias("cengine_batch_instr.so")
    so.ssm_decode_step.argtypes = [cf] * 9 + [ci] * 7
    so.ssm_layer_fused.argtypes = [cf] * 10 + [cu, ci, ci, ci, cu, ci, ci, ci] + [ci] * 7
    return so


def test_ssm_decode_step_matches_reference_c(ce):
    ro = dict(np.load(os.path.join(G, "ref_ops.npz")))
    B, N, inner, groups, ss, dtr = (int(v) for v in ro["ssm_dims"])
    interm = np.zeros(B * inner, np.float32)
    state = ro["ssm_state_in"].copy()
    norm = np.ones(ss, np.float32)
    ce.ssm_decode_step(p(ro["ssm_x"]), p(interm), p(ro["ssm_conv"]), p(ro["ssm_a"]), p(ro["ssm_dt"]),
                       p(ro["ssm_alpha"]), p(ro["ssm_beta"]), p(norm), p(state), B, N, inner, groups, ss, 4, dtr)
    assert O.rel_l2(interm, ro["ssm_interm"]) < 1e-5
    assert O.rel_l2(state, ro["ssm_state_out"]) < 1e-5


def engine_case(seed, B=10, N=2048, inner=4096, groups=32, ss=128, dtr=32):
    rng = np.random.default_rng(seed)
    return dict(
        x=rng.standard_normal(B * N).astype(np.float32),
        conv=(rng.standard_normal(4 * 2 * inner) * 0.5).astype(np.float32),
        a=-rng.uniform(0, 1, groups).astype(np.float32),
        dt=rng.standard_normal(groups).astype(np.float32),
        alpha=(rng.standard_normal(groups * dtr) * 0.1).astype(np.float32),
        beta=(rng.standard_normal(groups * dtr) * 0.1).astype(np.float32),
        state=rng.standard_normal(groups * ss).astype(np.float32),
        dims=(B, N, inner, groups, ss, dtr))


def test_ssm_decode_step_engine_dims(ce):
    c = engine_case(1)
    B, N, inner, groups, ss, dtr = c["dims"]
    interm = np.zeros(B * inner, np.float32)
    state = c["state"].copy()
    ce.ssm_decode_step(p(c["x"]), p(interm), p(c["conv"]), p(c["a"]), p(c["dt"]), p(c["alpha"]), p(c["beta"]),
                       p(np.ones(ss, np.float32)), p(state), B, N, inner, groups, ss, 4, dtr)
    ei, es = O.ssm_decode_step(c["x"], c["conv"], c["a"], c["dt"], c["alpha"], c["beta"], c["state"], B, N, inner,
                               groups, ss, dtr)
    assert O.rel_l2(interm, ei.reshape(-1)) < TOL
    assert O.rel_l2(state, es.reshape(-1)) < TOL


def test_ssm_layer_fused(ce):
    c = engine_case(2, B=3)
    B, N, inner, groups, ss, dtr = c["dims"]
    rng = np.random.default_rng(7)
    wg = F.quantize(F.Q8_0, (rng.standard_normal(inner * N) * 0.02).astype(np.float32))
    wo = F.quantize(F.Q4_K, (rng.standard_normal(N * inner) * 0.02).astype(np.float32))
    res = rng.standard_normal(B * N).astype(np.float32)
    out = np.zeros(B * N, np.float32)
    state = c["state"].copy()
    ce.ssm_layer_fused(p(c["x"]), p(res), p(out), p(c["conv"]), p(c["a"]), p(c["dt"]), p(c["alpha"]), p(c["beta"]),
                       p(np.ones(ss, np.float32)), p(state), wg.ctypes.data_as(cu), inner, N, F.Q8_0,
                       wo.ctypes.data_as(cu), N, inner, F.Q4_K, B, N, inner, groups, ss, 4, dtr)
    ei, es = O.ssm_decode_step(c["x"], c["conv"], c["a"], c["dt"], c["alpha"], c["beta"], c["state"], B, N, inner,
                               groups, ss, dtr)
    gate = O.gemv(wg, F.Q8_0, c["x"], inner, N)
    oproj = O.gemv(wo, F.Q4_K, (gate.astype(np.float64) * ei).astype(np.float32), N, inner)
    exp = res.reshape(B, N) + oproj
    assert O.rel_l2(out.reshape(B, N), exp) < TOL
    assert O.rel_l2(state, es.reshape(-1)) < TOL
