"""GPU parity of the row/elementwise ops (RMSNorm, SiLU, SwiGLU, residual add,
softmax, RoPE) through the reference-named simd_ops.so / combined_engine.so
entry points and the mlq_* C-ABI, against the oracle restatement.  These are
fp32 elementwise ops: tolerance is a few ulps (rtol 2e-6 .. 1e-5)."""
import ctypes

import numpy as np
import pytest

from oracle import ops as O

pytestmark = pytest.mark.gpu

cf = ctypes.POINTER(ctypes.c_float)


def p(a):
    return a.ctypes.data_as(cf)


@pytest.fixture(scope="module")
def libs(cuda_device):
    from mojollama_b200 import load_alias
    simd = load_alias("simd_ops.so")
    simd.rms_norm.argtypes = [cf, cf, cf, ctypes.c_int, ctypes.c_float]
    simd.silu.argtypes = [cf, cf, ctypes.c_int]
    simd.residual_add.argtypes = [cf, cf, cf, ctypes.c_int]
    simd.softmax.argtypes = [cf, ctypes.c_int]
    simd.apply_rope.argtypes = [cf, cf] + [ctypes.c_int] * 4 + [ctypes.c_float]
    eng = load_alias("combined_engine.so")
    eng.rms_norm.argtypes = [cf, cf, cf, ctypes.c_int]
    eng.silu.argtypes = [cf, ctypes.c_int]
    eng.softmax.argtypes = [cf, ctypes.c_int]
    eng.rope_init.argtypes = [cf, cf] + [ctypes.c_int] * 3
    return simd, eng, cuda_device


@pytest.mark.parametrize("n", [1, 7, 2048, 2880, 5003])
def test_rms_norm_both_signatures(libs, n):
    simd, eng, _ = libs
    rng = np.random.default_rng(n)
    x = (rng.standard_normal(n) * 3).astype(np.float32)
    w = rng.uniform(0.5, 1.5, n).astype(np.float32)
    out = np.zeros(n, np.float32)
    simd.rms_norm(p(out), p(x), p(w), n, 1e-6)
    np.testing.assert_allclose(out, O.rms_norm(x, w, 1e-6)[0], rtol=2e-6, atol=1e-7)
    out2 = np.zeros(n, np.float32)
    eng.rms_norm(p(x), p(w), p(out2), n)          # eps fixed 1e-5, argument order (x, w, out)
    np.testing.assert_allclose(out2, O.rms_norm(x, w, 1e-5)[0], rtol=2e-6, atol=1e-7)


def test_rms_norm_sanitize_and_rows(libs):
    _, _, lib = libs
    rng = np.random.default_rng(0)
    x = (rng.standard_normal((4, 512)) * 600).astype(np.float32)
    x[1, 3] = np.nan
    x[2, 7] = 1e9
    w = np.ones(512, np.float32)
    out = np.zeros_like(x)
    res = np.zeros_like(x)
    assert lib.mlq_rms_norm(out.ctypes.data, x.ctypes.data, w.ctypes.data, 4, 512, 1e-5, 1, res.ctypes.data) == 0
    exp, clamped = O.rms_norm(x, w, 1e-5, sanitize=True)
    np.testing.assert_allclose(out, exp, rtol=2e-6, atol=1e-6)
    np.testing.assert_array_equal(res, clamped)


@pytest.mark.parametrize("n", [5, 8, 1000, 4099])
def test_silu_modes(libs, n):
    simd, eng, _ = libs
    x = (np.random.default_rng(n).standard_normal(n) * 4).astype(np.float32)
    out = np.zeros(n, np.float32)
    simd.silu(p(out), p(x), n)                       # Pade body + exact tail
    np.testing.assert_allclose(out, O.silu(x, 1), rtol=1e-5, atol=1e-6)
    y = x.copy()
    eng.silu(p(y), n)                                # exact, in place
    np.testing.assert_allclose(y, O.silu(x, 0), rtol=1e-5, atol=1e-6)


def test_swiglu_and_add(libs):
    _, _, lib = libs
    rng = np.random.default_rng(1)
    g = (rng.standard_normal(3000) * 50).astype(np.float32)
    u = rng.standard_normal(3000).astype(np.float32)
    h = np.zeros(3000, np.float32)
    assert lib.mlq_swiglu(h.ctypes.data, g.ctypes.data, u.ctypes.data, 3000) == 0
    np.testing.assert_allclose(h, O.swiglu(g, u), rtol=1e-5, atol=1e-6)
    simd, _, _ = libs
    o = np.zeros(3000, np.float32)
    simd.residual_add(p(o), p(g), p(u), 3000)
    np.testing.assert_array_equal(o, g + u)


@pytest.mark.parametrize("n", [1, 33, 4096])
def test_softmax(libs, n):
    simd, eng, _ = libs
    x = (np.random.default_rng(n).standard_normal(n) * 5).astype(np.float32)
    y = x.copy()
    simd.softmax(p(y), n)
    np.testing.assert_allclose(y, O.softmax(x), rtol=1e-5, atol=1e-8)
    y = x.copy()
    eng.softmax(p(y), n)
    np.testing.assert_allclose(y, O.softmax(x), rtol=1e-5, atol=1e-8)


def test_apply_rope_interleaved(libs):
    simd, _, _ = libs
    nh, nkh, hd, pos = 32, 4, 64, 77
    rng = np.random.default_rng(2)
    q = rng.standard_normal(nh * hd).astype(np.float32)
    k = rng.standard_normal(nkh * hd).astype(np.float32)
    q2, k2 = q.copy(), k.copy()
    simd.apply_rope(p(q2), p(k2), nh, nkh, hd, pos, 10000.0)
    eq, ek = O.rope_interleaved(q, k, nh, nkh, hd, pos, 10000.0)
    np.testing.assert_allclose(q2, eq, rtol=1e-4, atol=2e-5)
    np.testing.assert_allclose(k2, ek, rtol=1e-4, atol=2e-5)


@pytest.mark.parametrize("hd,rope_dim", [(64, 64), (128, 128), (256, 64)])
def test_rope_tables_and_neox(libs, hd, rope_dim):
    _, eng, lib = libs
    max_ctx = 4096
    c = np.zeros(max_ctx * rope_dim // 2, np.float32)
    s = np.zeros_like(c)
    eng.rope_init(p(c), p(s), max_ctx, hd, rope_dim)
    ec, es = O.rope_tables(max_ctx, hd, rope_dim)
    np.testing.assert_allclose(c.reshape(ec.shape), ec, atol=2e-7)
    np.testing.assert_allclose(s.reshape(es.shape), es, atol=2e-7)
    nh, rows = 8, 3
    rng = np.random.default_rng(hd)
    buf = rng.standard_normal((rows, nh * hd)).astype(np.float32)
    pos = np.array([0, 17, 4095], np.int32)
    out = buf.copy()
    assert lib.mlq_rope_neox(out.ctypes.data, rows, 0, nh, hd, pos.ctypes.data, 0, c.ctypes.data, s.ctypes.data,
                             rope_dim, max_ctx) == 0
    for r in range(rows):
        exp = O.rope_neox(buf[r], nh, hd, pos[r], ec, es, rope_dim)
        np.testing.assert_allclose(out[r], exp, rtol=1e-5, atol=1e-5)
