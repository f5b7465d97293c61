"""GPU parity of the MXFP4 GEMV on the block-scaled tensor cores (tcgen05.mma kind::mxf4,
E8M0 scales; the reference's mxfp4 matmuls behind quant_matmul_omp type 39,
quant_kernels_omp.c:502-732, in the GGUF MXFP4 layout) against the fp64 oracle.

Tolerance: relative L2 <= 1e-3.  The weights enter the MMA exactly (their own E2M1 codes
and E8M0 scales); the activations as 8 residual E2M1 planes with per-32-element scales
(|error| <~ 4^-8 of the block maximum); products exact, sums fp32.  Covered: ragged row
tiles, K from one 512-element chunk to 8192, 1-8 activation rows per weight pass and
batches split into several passes, activations spanning 1e-6..1e6 within a row, zero rows,
a non-finite activation, and row-tile counts whose chunks do not divide evenly over the
SMs (stream-K: tiles split between CTAs, partial sums added in a fixed order)."""
import ctypes

import numpy as np
import pytest

from oracle import formats as F
from oracle import ops as O

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _mm(lib, torch, w, x, n, k):
    m = x.shape[0]
    dw = torch.from_numpy(w).cuda()
    dx = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    do = torch.full((m * n,), float("nan"), device="cuda")
    torch.cuda.synchronize()
    l0 = lib.mlq_launch_count()
    rc = lib.mlq_matmul(ctypes.c_void_p(dw.data_ptr()), F.MXFP4, ctypes.c_void_p(dx.data_ptr()),
                        ctypes.c_void_p(do.data_ptr()), n, k, m)
    assert rc == 0, lib.mlq_last_error_message()
    torch.cuda.synchronize()
    return do.cpu().numpy().reshape(m, n), lib.mlq_launch_count() - l0


def _weights(rng, n, k):
    return F.quantize(F.MXFP4, (rng.standard_normal(n * k) * 0.02).astype(np.float32))


@pytest.mark.parametrize("n,k,m", [(512, 2048, 1), (1000, 1024, 1), (300, 512, 1), (4096, 2048, 1),
                                   (130, 4096, 1), (2000, 8192, 1), (256, 2048, 2), (200, 2048, 3),
                                   (640, 1024, 8), (333, 2048, 4), (129, 512, 7), (20000, 1024, 1),
                                   (9000, 2048, 2)])
def test_mxf4_tc_matches_oracle(cuda_device, n, k, m):
    import torch
    rng = np.random.default_rng(n * 7 + k + m)
    w = _weights(rng, n, k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    got, launches = _mm(cuda_device, torch, w, x, n, k)
    want = O.gemv(w, F.MXFP4, x, n, k)
    assert O.rel_l2(got, want) < TOL, O.rel_l2(got, want)
    assert launches == 1, launches          # one tensor-core launch (it encodes the planes itself)


def test_mxf4_tc_batch_in_passes(cuda_device):
    """B = 4 at K = 4096 runs as two passes of 2 activation rows over the same weights (from 5
    rows a batch that needs more than one pass goes to the tensor-core GEMM)."""
    import torch
    n, k, m = 777, 4096, 4
    rng = np.random.default_rng(3)
    w = _weights(rng, n, k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    got, launches = _mm(cuda_device, torch, w, x, n, k)
    want = O.gemv(w, F.MXFP4, x, n, k)
    for t in range(m):
        assert O.rel_l2(got[t], want[t]) < TOL, t
    assert launches == 2, launches


def test_mxf4_tc_dynamic_range(cuda_device):
    """Elements from 1e-6 to 1e6 inside one row, a zero row and a row of tiny values."""
    import torch
    n, k, m = 384, 1024, 3
    rng = np.random.default_rng(11)
    w = _weights(rng, n, k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    x[0] *= np.logspace(-6, 6, k, dtype=np.float32)[rng.permutation(k)]
    x[1] = 0.0
    x[2] *= 1e-30
    got, _ = _mm(cuda_device, torch, w, x, n, k)
    want = O.gemv(w, F.MXFP4, x, n, k)
    assert O.rel_l2(got[0], want[0]) < TOL, O.rel_l2(got[0], want[0])
    assert np.all(got[1] == 0.0)
    assert O.rel_l2(got[2], want[2]) < TOL, O.rel_l2(got[2], want[2])


def test_mxf4_tc_nonfinite_activation(cuda_device):
    """A NaN activation makes every output of its row NaN (as W x does); other rows stay exact."""
    import torch
    n, k, m = 256, 1024, 2
    rng = np.random.default_rng(12)
    w = _weights(rng, n, k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    x[0, 100] = np.nan
    got, _ = _mm(cuda_device, torch, w, x, n, k)
    assert np.all(np.isnan(got[0]))
    want = O.gemv(w, F.MXFP4, x[1:], n, k)
    assert O.rel_l2(got[1], want[0]) < TOL
