"""Mamba-2 decode step: the oracle (oracle/mamba2.py) pinned to an independent
implementation, and the library's kernels (mojollama_b200/csrc/mamba2.cu) against the
oracle.

CPU: the oracle run over the golden tokens of tests/golden/mamba2.npz (Hugging Face
transformers 5.5.0's plain-torch Mamba2Mixer in float64: its chunked SSD prefill path for
the first token, its recurrent decode path after) reproduces every step's output and the
final conv / SSM states.
GPU: mlq_mamba2_step and mlq_mamba2_layer through the C-ABI against the oracle, on the
golden model and at config 5's head shape (16 heads x 128, state 128, conv width 4,
A = -exp(U[0, 1]), dt from N(0, 1)), several steps in a row, states in place.
Bars: relative L2 <= 1e-3 per output (fp32 arithmetic, fp64 oracle); the golden pin
holds to 1e-6 (the oracle in float64 against transformers in float64)."""
import ctypes
import os

import numpy as np
import pytest

from oracle import mamba2 as M2
from oracle import ops as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "mamba2.npz")
TOL = 1e-3


def _golden():
    g = np.load(GOLD)
    H, P, S, G, K = (int(v) for v in g["dims"])
    p = dict(H=H, P=P, S=S, G=G, conv_w=g["conv_w"], conv_b=g["conv_b"], A_log=g["A_log"], dt_bias=g["dt_bias"],
             D=g["D"], norm_w=g["norm_w"])
    return g, p, K


def test_oracle_matches_transformers_mamba2():
    g, p, K = _golden()
    T, B, hidden = g["u"].shape
    conv_dim = p["H"] * p["P"] + 2 * p["G"] * p["S"]
    cs = np.zeros((B, conv_dim, K), np.float64)
    ss = np.zeros((B, p["H"], p["P"], p["S"]), np.float64)
    for t in range(T):
        out = M2.mamba2_layer_step(g["u"][t], g["W_in"], g["W_out"], cs, ss, p, eps=float(g["eps"][0]))
        assert O.rel_l2(out, g["out"][t]) < 1e-6, t
    assert O.rel_l2(cs, g["conv_state"]) < 1e-12
    assert O.rel_l2(ss, g["ssm_state"]) < 1e-6


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def _vp(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


@pytest.mark.gpu
def test_mamba2_layer_matches_golden_model(cuda_device):
    import torch
    lib = cuda_device
    g, p, K = _golden()
    T, B, hidden = g["u"].shape
    H, P, S, G = p["H"], p["P"], p["S"], p["G"]
    conv_dim = H * P + 2 * G * S
    cs = torch.zeros((B, conv_dim, K), device="cuda")
    ss = torch.zeros((B, H, P, S), device="cuda")
    cs_o = np.zeros((B, conv_dim, K), np.float32)
    ss_o = np.zeros((B, H, P, S), np.float32)
    w_in, w_out = _dev(g["W_in"]), _dev(g["W_out"])
    prm = [_dev(p[k]) for k in ("conv_w", "conv_b", "A_log", "dt_bias", "D", "norm_w")]
    for t in range(T):
        u = _dev(g["u"][t])
        out = torch.full((B, hidden), float("nan"), device="cuda")
        rc = lib.mlq_mamba2_layer(_vp(u), B, hidden, _vp(w_in), 0, _vp(w_out), 0, _vp(cs), *[_vp(x) for x in prm],
                                  _vp(ss), _vp(out), H, P, S, G, K, ctypes.c_float(float(g["eps"][0])), 0)
        assert rc == 0, lib.mlq_last_error_message()
        torch.cuda.synchronize()
        want = M2.mamba2_layer_step(g["u"][t], g["W_in"], g["W_out"], cs_o, ss_o, p, eps=float(g["eps"][0]))
        got = out.cpu().numpy()
        assert O.rel_l2(got, want) < TOL, (t, O.rel_l2(got, want))
        assert O.rel_l2(got, g["out"][t]) < TOL
    assert O.rel_l2(ss.cpu().numpy(), ss_o) < TOL
    assert O.rel_l2(cs.cpu().numpy(), cs_o) < 1e-6


@pytest.mark.gpu
@pytest.mark.parametrize("B,H,P,S,G,gated,norm_groups", [
    (10, 16, 128, 128, 1, True, 1),      # config 5's SSM layer shape, B = 10 sequences
    (3, 16, 128, 128, 2, True, 2),       # grouped B/C and mamba_ssm's per-group norm
    (4, 8, 64, 64, 1, False, 0),         # no gate, no norm
    (1, 24, 64, 16, 4, True, 1),         # small state
])
def test_mamba2_step_matches_oracle(cuda_device, B, H, P, S, G, gated, norm_groups):
    import torch
    lib = cuda_device
    rng = np.random.default_rng(B * 1000 + H + S)
    d_inner, K = H * P, 4
    conv_dim = d_inner + 2 * G * S
    conv_w = (rng.standard_normal((conv_dim, K)) * 0.5).astype(np.float32)
    conv_b = (rng.standard_normal(conv_dim) * 0.1).astype(np.float32)
    A_log = rng.random(H).astype(np.float32)                      # A = -exp(U[0, 1])
    dt_bias = (rng.standard_normal(H) * 0.5).astype(np.float32)
    D = rng.standard_normal(H).astype(np.float32)
    norm_w = (1 + 0.1 * rng.standard_normal(d_inner)).astype(np.float32) if norm_groups else None
    norm_group = d_inner // norm_groups if norm_groups else 0
    cs_o = (rng.standard_normal((B, conv_dim, K))).astype(np.float32)
    ss_o = (rng.standard_normal((B, H, P, S)) * 0.3).astype(np.float32)
    cs, ss = _dev(cs_o), _dev(ss_o)
    prm = [_dev(conv_w), _dev(conv_b), _dev(A_log), _dev(dt_bias), _dev(D),
           _dev(norm_w) if norm_w is not None else None]
    for step in range(3):
        xbc = rng.standard_normal((B, conv_dim)).astype(np.float32)
        z = rng.standard_normal((B, d_inner)).astype(np.float32) if gated else None
        dt = rng.standard_normal((B, H)).astype(np.float32)              # dt softplus of N(0, 1) + bias
        y = torch.full((B, d_inner), float("nan"), device="cuda")
        # device copies held in names until the call has run (a temporary's memory could be
        # handed to the next allocation before the kernels read it)
        dx, ddt = _dev(xbc), _dev(dt)
        dz = _dev(z) if gated else None
        rc = lib.mlq_mamba2_step(_vp(dx), _vp(dz), _vp(ddt), _vp(cs), *[_vp(x) for x in prm], _vp(ss),
                                 _vp(y), B, H, P, S, G, K, ctypes.c_float(1e-5), norm_group)
        assert rc == 0, lib.mlq_last_error_message()
        want = M2.mamba2_step(xbc, z, dt, cs_o, conv_w, conv_b, A_log, dt_bias, D, norm_w, ss_o, H, P, S, G,
                              eps=1e-5, norm_group=norm_group or None)
        torch.cuda.synchronize()
        assert O.rel_l2(y.cpu().numpy(), want) < TOL, (step, O.rel_l2(y.cpu().numpy(), want))
    assert O.rel_l2(ss.cpu().numpy(), ss_o) < TOL
    assert np.array_equal(cs.cpu().numpy(), cs_o)


@pytest.mark.gpu
def test_mamba2_rejects_bad_shapes(cuda_device):
    lib = cuda_device
    f = np.zeros(64, np.float32)
    # heads not a multiple of groups
    rc = lib.mlq_mamba2_step(f.ctypes.data, None, f.ctypes.data, f.ctypes.data, f.ctypes.data, None, f.ctypes.data,
                             f.ctypes.data, None, None, f.ctypes.data, f.ctypes.data, 1, 3, 8, 8, 2, 4,
                             ctypes.c_float(1e-5), 0)
    assert rc == 1
