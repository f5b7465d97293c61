"""GPU parity of the tensor-core (tcgen05) quantized GEMM that serves batches of >= 5
tokens (the reference's *_batch_matmul math, cengine_batch_instr.c:68-534), against the
fp64 oracle: weights dequantized exactly, x [M][K] fp32, out [M][N] fp32.

Tolerance: relative L2 <= 1e-3 (the kernel rounds weights and activations once to fp16
with a power-of-two scale per token; products and sums are fp32).  Covered: every format
the tensor-core path takes, ragged row tiles (N not a multiple of 128), token counts that
are not multiples of the token tile (5 and 10 tokens in a 16-token tile), several tiles of tokens, activations with a large
dynamic range, and the reference-named batch entry points."""
import ctypes

import numpy as np
import pytest

from oracle import formats as F
from oracle import ops as O

pytestmark = pytest.mark.gpu
TOL = 1e-3
TC_FORMATS = [F.Q8_0, F.Q4_0, F.Q4_1, F.Q5_0, F.Q4_K, F.Q5_K, F.Q6_K, F.MXFP4]


def _mm(lib, torch, w, qt, x, n, k):
    m = x.shape[0]
    dw = torch.from_numpy(w).cuda()
    dx = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    do = torch.empty(m * n, device="cuda")
    rc = lib.mlq_matmul(ctypes.c_void_p(dw.data_ptr()), qt, ctypes.c_void_p(dx.data_ptr()),
                        ctypes.c_void_p(do.data_ptr()), n, k, m)
    assert rc == 0, lib.mlq_last_error_message()
    torch.cuda.synchronize()
    return do.cpu().numpy().reshape(m, n)


@pytest.mark.parametrize("qt", TC_FORMATS, ids=lambda q: F.NAMES[q])
@pytest.mark.parametrize("n,k,m", [(384, 512, 16), (200, 256, 17), (1000, 2048, 64), (130, 768, 100),
                                   (256, 512, 256), (512, 2048, 5), (300, 1024, 10)])
def test_tc_gemm_matches_oracle(cuda_device, qt, n, k, m):
    import torch
    rng = np.random.default_rng(qt * 1000 + n + m)
    w = F.quantize(qt, (rng.standard_normal(n * k) * 0.02).astype(np.float32))
    x = rng.standard_normal((m, k)).astype(np.float32)
    got = _mm(cuda_device, torch, w, qt, x, n, k)
    want = O.gemv(w, qt, x, n, k)
    assert O.rel_l2(got, want) < TOL, O.rel_l2(got, want)


@pytest.mark.parametrize("qt", [F.Q8_0, F.Q4_0, F.Q4_1, F.Q5_0, F.MXFP4], ids=lambda q: F.NAMES[q])
@pytest.mark.parametrize("n,k,m", [(2880, 2880, 16), (300, 2880, 64), (129, 96, 16), (257, 1312, 40)])
def test_tc_gemm_block32_ragged_k(cuda_device, qt, n, k, m):
    """32-element block formats with K not a multiple of the 256-element chunk (the last
    chunk partly empty) and rows that do not start on 16 bytes (K = 2880: 3060-byte Q8_0
    rows; MXFP4's 17-byte blocks), down to a single partial chunk (K = 96); the last row's
    last piece ends at the end of the weight buffer."""
    import torch
    rng = np.random.default_rng(qt * 7 + n + k)
    w = F.quantize(qt, (rng.standard_normal(n * k) * 0.02).astype(np.float32))
    x = rng.standard_normal((m, k)).astype(np.float32)
    got = _mm(cuda_device, torch, w, qt, x, n, k)
    want = O.gemv(w, qt, x, n, k)
    assert O.rel_l2(got, want) < TOL, O.rel_l2(got, want)


@pytest.mark.parametrize("n,k,m", [(300, 2048, 16), (257, 2880, 64)])
def test_tc_gemm_mxfp4_any_block_scale(cuda_device, n, k, m):
    """MXFP4 blocks with random E8M0 scales (2^-128 .. 2^127): every chunk's product is
    formed relative to its rows' largest block scale and scaled back in fp32, so no scale
    leaves the fp16 operand's range"""
    import torch
    rng = np.random.default_rng(n + k + m)
    w = F.random_blocks(F.MXFP4, n * k, rng)
    x = rng.standard_normal((m, k)).astype(np.float32)
    got = _mm(cuda_device, torch, w, F.MXFP4, x, n, k)
    want = O.gemv(w, F.MXFP4, x, n, k)
    assert np.isfinite(got).all()
    assert O.rel_l2(got, want) < TOL, O.rel_l2(got, want)


def test_tc_gemm_per_token_scale(cuda_device):
    """Tokens whose magnitudes differ by 1e8 (and a zero token) keep their own precision."""
    import torch
    n, k, m = 256, 512, 24
    rng = np.random.default_rng(5)
    w = F.quantize(F.Q8_0, (rng.standard_normal(n * k) * 0.02).astype(np.float32))
    x = rng.standard_normal((m, k)).astype(np.float32)
    x *= np.logspace(-4, 4, m, dtype=np.float32)[:, None]
    x[3] = 0.0
    got = _mm(cuda_device, torch, w, F.Q8_0, x, n, k)
    want = O.gemv(w, F.Q8_0, x, n, k)
    for t in range(m):
        assert O.rel_l2(got[t], want[t]) < TOL, t
    assert np.all(got[3] == 0.0)


@pytest.mark.parametrize("name,qt", [("q8_0", F.Q8_0), ("q4_0", F.Q4_0), ("q4_k", F.Q4_K)])
def test_tc_through_batch_matmul_abi(cuda_device, name, qt):
    """The reference-named x [B][nc] -> out [B][n_rows] entry with host buffers, B = 32."""
    from mojollama_b200.kernels import load_kernels
    kern = load_kernels().kern
    n, k, b = 512, 1024, 32
    rng = np.random.default_rng(qt)
    w = F.quantize(qt, (rng.standard_normal(n * k) * 0.02).astype(np.float32))
    x = rng.standard_normal((b, k)).astype(np.float32)
    out = np.zeros(b * n, np.float32)
    getattr(kern, f"{name}_batch_matmul")(w.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)),
                                          x.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                          out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), n, k, b)
    want = O.gemv(w, qt, x, n, k)
    assert O.rel_l2(out.reshape(b, n), want) < TOL


def test_q6k_batch_takes_tensor_cores(cuda_device):
    """Q6_K at 64 tokens runs as one activation conversion + one tensor-core launch (not
    8 passes of the 8-row GEMV), rows of 630 bytes (K = 768) included."""
    import torch
    lib = cuda_device
    for n, k in [(1000, 2048), (300, 768)]:
        rng = np.random.default_rng(n + k)
        w = F.quantize(F.Q6_K, (rng.standard_normal(n * k) * 0.02).astype(np.float32))
        x = rng.standard_normal((64, k)).astype(np.float32)
        dw = torch.from_numpy(w).cuda()
        dx = torch.from_numpy(x).cuda()
        do = torch.empty(64 * n, device="cuda")
        torch.cuda.synchronize()
        l0 = lib.mlq_launch_count()
        assert lib.mlq_matmul(ctypes.c_void_p(dw.data_ptr()), F.Q6_K, ctypes.c_void_p(dx.data_ptr()),
                              ctypes.c_void_p(do.data_ptr()), n, k, 64) == 0
        torch.cuda.synchronize()
        assert lib.mlq_launch_count() - l0 == 2
        got = do.cpu().numpy().reshape(64, n)
        assert O.rel_l2(got, O.gemv(w, F.Q6_K, x, n, k)) < TOL
