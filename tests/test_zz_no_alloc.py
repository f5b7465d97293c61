"""mlq_matmul_q8act_noalloc: the Q8_0-activation matmul for callers that cannot let a
library allocate device memory (their HBM belongs to their own allocator, or their
decode loop must not hit cudaMalloc/cudaFree).  It keeps its scratch in a fixed
device array instead of allocating.

Checked through the C-ABI on two calls in a row that share the scratch array: against
the oracle (the weights times the dequantised Q8_0 activations, float64) and against
the existing entry point mlq_matmul_q8act, within the tolerance of the other matmul
tests.  B = 3 runs the few-row GEMV; B = 32 at 2048 columns fills the array exactly
(65536 elements) and is the batch size at which the allocating entry point takes the
tensor-core GEMM, which needs scratch and therefore steps aside here.  After every call
mlq_noalloc_status must report that no device-side wait gave up.

This file is collected last on purpose (tests/test_zz_*), and passes both alone in a
fresh process and after the rest of the suite."""
import ctypes

import numpy as np
import pytest

from mojollama_b200 import core
from oracle import formats as F
from oracle import ops as O

pytestmark = pytest.mark.gpu

TOL = 1e-3


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("b", [3, 32])
@pytest.mark.parametrize("qt", [F.Q4_K, F.Q8_0, F.MXFP4])
def test_noalloc_matches_oracle_and_existing_entry_point_on_two_calls(cuda_device, qt, b):
    import torch
    lib = core()
    stream = torch.cuda.current_stream().cuda_stream
    lib.mlq_set_stream(stream)
    n, k = 1536, 2048
    rng = np.random.default_rng(qt * 100 + b)
    w_host = F.quantize(qt, (rng.standard_normal(n * k) * 0.02).astype(np.float32))
    w = _dev(w_host)
    for call in range(2):                      # two calls in a row share the scratch array
        x = rng.standard_normal(b * k).astype(np.float32) * (1 + call)
        xq_host = F.quantize_q8_0(x)
        xq = _dev(xq_host)
        got = torch.full((b, n), float("nan"), device="cuda")
        want = torch.zeros((b, n), device="cuda")
        rc = lib.mlq_matmul_q8act_noalloc(w.data_ptr(), qt, xq.data_ptr(), got.data_ptr(), n, k, b,
                                          ctypes.c_void_p(stream))
        assert rc == 0, lib.mlq_last_error_message()
        assert lib.mlq_noalloc_status(ctypes.c_void_p(stream)) == 0, lib.mlq_last_error_message()
        assert lib.mlq_matmul_q8act(w.data_ptr(), qt, xq.data_ptr(), want.data_ptr(), n, k, b) == 0
        torch.cuda.synchronize()
        g, e = got.cpu().numpy(), want.cpu().numpy()
        assert np.all(np.isfinite(g))
        x_dq = F.dequantize(F.Q8_0, xq_host, b * k).reshape(b, k)
        ref = O.gemv(w_host, qt, x_dq, n, k)
        assert O.rel_l2(g, ref) < TOL, (call, "oracle", O.rel_l2(g, ref))
        assert O.rel_l2(g, e) < TOL, (call, "mlq_matmul_q8act", O.rel_l2(g, e))


def test_noalloc_rejects_what_it_cannot_do(cuda_device):
    import torch
    lib = core()
    n, k = 64, 4096
    w = _dev(F.quantize(F.Q8_0, np.zeros(n * k, np.float32)))
    out = torch.full((17, n), 7.0, device="cuda")
    xq = torch.zeros(17 * k // 32 * 34, dtype=torch.uint8, device="cuda")
    # 17 * 4096 > 65536 fp32 scratch elements: refused before any launch
    rc = lib.mlq_matmul_q8act_noalloc(w.data_ptr(), F.Q8_0, xq.data_ptr(), out.data_ptr(), n, k, 17, None)
    assert rc == 6 and b"exceeds" in lib.mlq_last_error_message()
    # a type the matmul does not know: refused with MLQ_ERR_TYPE before any launch
    rc = lib.mlq_matmul_q8act_noalloc(w.data_ptr(), 77, xq.data_ptr(), out.data_ptr(), n, k, 1, None)
    assert rc == 2
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())
    # host pointers are refused: this entry point copies nothing
    host_out = np.zeros(n, np.float32)
    rc = lib.mlq_matmul_q8act_noalloc(w.data_ptr(), F.Q8_0, xq.data_ptr(), host_out.ctypes.data, n, k, 1, None)
    assert rc == 1
    assert lib.mlq_noalloc_status(None) == 0
