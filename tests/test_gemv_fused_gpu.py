"""GPU parity of the batch engine's decode GEMV (mlq_gemv_fused: packed activation rows,
segmented matrices, residual and SiLU-mul epilogues) against the oracle GEMV:
  mode 0  out_i = x W_i^T                       (q / k / v of one type in one launch)
  mode 1  out_i = res_i + x W_i^T               (o / down projection + residual add)
  mode 2  out_0 = silu(x W_0^T) * (x W_1^T)     (gate / up + SiLU-mul, exact silu)
cengine_batch_instr.c:1349-1351, 1409, 1463-1467.  Every format, B = 1..8, rows that are
not a multiple of the tile, rows shorter than a warp's 32 units (lane groups) and rows
whose length is not a multiple of 128 bytes.  Tolerance: relative L2 <= 1e-3 per row."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import formats as F
from oracle import ops as O

pytestmark = pytest.mark.gpu
TOL = 1e-3
FORMATS = [F.Q4_0, F.Q4_1, F.Q5_0, F.Q8_0, F.Q4_K, F.Q5_K, F.Q6_K, F.MXFP4]


def _mat(qt, rows, K, rng):
    raw = F.random_blocks(qt, rows * K, rng)
    return raw, F.dequantize(qt, raw, rows * K).astype(np.float64).reshape(rows, K)


def _call(lib, qt, mats, outs, res, mode, x):
    n = len(mats)
    B, K = x.shape
    arr_p = (ctypes.c_void_p * n)
    W = arr_p(*[m.data_ptr() for m in mats])
    rows = (ctypes.c_int * n)(*[o.shape[1] for o in outs])
    out = arr_p(*[o.data_ptr() for o in outs])
    rs = arr_p(*[r.data_ptr() for r in res]) if res else None
    dx = torch.from_numpy(x).cuda()
    rc = lib.mlq_gemv_fused(qt, n, W, rows, out, rs, mode, ctypes.c_void_p(dx.data_ptr()), B, K)
    assert rc == 0, lib.mlq_last_error_message()
    torch.cuda.synchronize()


def _check(got, want):
    for b in range(want.shape[0]):
        assert O.rel_l2(got[b], want[b]) < TOL, (b, O.rel_l2(got[b], want[b]))


@pytest.mark.parametrize("qt", FORMATS)
@pytest.mark.parametrize("B", [1, 3, 4, 8])
def test_segments_qkv(cuda_device, qt, B):
    """three matrices of one type, one input: 80 / 16 / 16 rows (ragged last tiles)"""
    rng = np.random.default_rng(qt * 10 + B)
    K = 512
    parts = [_mat(qt, r, K, rng) for r in (80, 16, 16)]
    x = rng.standard_normal((B, K)).astype(np.float32)
    mats = [torch.from_numpy(p[0]).cuda() for p in parts]
    outs = [torch.full((B, p[1].shape[0]), float("nan"), device="cuda") for p in parts]
    _call(cuda_device, qt, mats, outs, None, 0, x)
    for o, p in zip(outs, parts):
        _check(o.cpu().numpy(), x.astype(np.float64) @ p[1].T)


@pytest.mark.parametrize("qt", FORMATS)
def test_residual(cuda_device, qt):
    rng = np.random.default_rng(qt)
    B, K, n = 4, 768, 100
    raw, Wm = _mat(qt, n, K, rng)
    x = rng.standard_normal((B, K)).astype(np.float32)
    r = rng.standard_normal((B, n)).astype(np.float32)
    out = torch.full((B, n), float("nan"), device="cuda")
    _call(cuda_device, qt, [torch.from_numpy(raw).cuda()], [out], [torch.from_numpy(r).cuda()], 1, x)
    _check(out.cpu().numpy(), r.astype(np.float64) + x.astype(np.float64) @ Wm.T)


@pytest.mark.parametrize("qt", FORMATS)
@pytest.mark.parametrize("B", [1, 2, 5])
def test_pair_silu(cuda_device, qt, B):
    rng = np.random.default_rng(qt * 3 + B)
    K, n = 256, 200
    g, Gm = _mat(qt, n, K, rng)
    u, Um = _mat(qt, n, K, rng)
    x = (rng.standard_normal((B, K)) * 4).astype(np.float32)
    out = torch.full((B, n), float("nan"), device="cuda")
    _call(cuda_device, qt, [torch.from_numpy(g).cuda(), torch.from_numpy(u).cuda()], [out, out], None, 2, x)
    xd = x.astype(np.float64)
    gv, uv = xd @ Gm.T, xd @ Um.T
    _check(out.cpu().numpy(), gv / (1 + np.exp(-gv)) * uv)


@pytest.mark.parametrize("qt,K", [(F.Q8_0, 64), (F.Q4_0, 96), (F.MXFP4, 2880), (F.Q6_K, 256)])
def test_short_and_odd_rows(cuda_device, qt, K):
    """2-unit rows (16 rows per warp pass), 96- and 2880-element rows (partial 128-byte groups)"""
    rng = np.random.default_rng(K)
    B, n = 6, 50
    raw, Wm = _mat(qt, n, K, rng)
    x = rng.standard_normal((B, K)).astype(np.float32)
    out = torch.full((B, n), float("nan"), device="cuda")
    _call(cuda_device, qt, [torch.from_numpy(raw).cuda()], [out], None, 0, x)
    _check(out.cpu().numpy(), x.astype(np.float64) @ Wm.T)


@pytest.mark.parametrize("B", [1, 4])
def test_config1_layer_shapes(cuda_device, B):
    """The config-1 (TinyLlama-1.1B shape, Q8_0) decode projections at their full sizes:
    q/k/v (2048 + 256 + 256 rows, K 2048) in one launch, o + residual (2048 x 2048),
    gate/up + SiLU-mul (5632 x 2048) and down + residual (2048 x 5632, the long rows)."""
    qt = F.Q8_0
    rng = np.random.default_rng(40 + B)
    N, FF, kv = 2048, 5632, 256
    x = rng.standard_normal((B, N)).astype(np.float32)
    xd = x.astype(np.float64)
    parts = [_mat(qt, r, N, rng) for r in (N, kv, kv)]
    outs = [torch.full((B, p[1].shape[0]), float("nan"), device="cuda") for p in parts]
    _call(cuda_device, qt, [torch.from_numpy(p[0]).cuda() for p in parts], outs, None, 0, x)
    for o, p in zip(outs, parts):
        _check(o.cpu().numpy(), xd @ p[1].T)
    raw, Wm = _mat(qt, N, N, rng)
    r = rng.standard_normal((B, N)).astype(np.float32)
    out = torch.full((B, N), float("nan"), device="cuda")
    _call(cuda_device, qt, [torch.from_numpy(raw).cuda()], [out], [torch.from_numpy(r).cuda()], 1, x)
    _check(out.cpu().numpy(), r.astype(np.float64) + xd @ Wm.T)
    g, Gm = _mat(qt, FF, N, rng)
    u, Um = _mat(qt, FF, N, rng)
    out = torch.full((B, FF), float("nan"), device="cuda")
    _call(cuda_device, qt, [torch.from_numpy(g).cuda(), torch.from_numpy(u).cuda()], [out, out], None, 2, x)
    gv, uv = xd @ Gm.T, xd @ Um.T
    _check(out.cpu().numpy(), gv / (1 + np.exp(-gv)) * uv)
    h = rng.standard_normal((B, FF)).astype(np.float32)
    raw, Wm = _mat(qt, N, FF, rng)
    out = torch.full((B, N), float("nan"), device="cuda")
    _call(cuda_device, qt, [torch.from_numpy(raw).cuda()], [out], [torch.from_numpy(r).cuda()], 1, h)
    _check(out.cpu().numpy(), r.astype(np.float64) + h.astype(np.float64) @ Wm.T)
