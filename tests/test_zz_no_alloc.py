"""mlq_matmul_q8act_noalloc: the Q8_0-activation matmul for callers that cannot let a
library allocate device memory (their HBM belongs to their own allocator, or their
decode loop must not hit cudaMalloc/cudaFree).  It keeps its scratch in a fixed
device array instead of allocating.  Checked through the C-ABI against the existing
entry point mlq_matmul_q8act, on two calls in a row that share the scratch.

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


@pytest.mark.parametrize("qt", [F.Q4_K, F.Q8_0, F.MXFP4])
def test_noalloc_matches_existing_entry_point_on_two_calls(cuda_device, qt):
    import torch
    lib = core()
    stream = torch.cuda.current_stream().cuda_stream
    lib.mlq_set_stream(stream)
    n, k, b = 1536, 2048, 3
    rng = np.random.default_rng(qt)
    w = _dev(F.quantize(qt, (rng.standard_normal(n * k) * 0.02).astype(np.float32)))
    for call in range(2):                      # two calls in a row share the scratch array
        x = rng.standard_normal(b * k).astype(np.float32) * (1 + call)
        xq = _dev(F.quantize_q8_0(x))
        got = torch.full((b, n), float("nan"), device="cuda")
        want = torch.zeros((b, n), device="cuda")
        rc = lib.mlq_matmul_q8act_noalloc(w.data_ptr(), qt, xq.data_ptr(), got.data_ptr(), n, k, b,
                                          ctypes.c_void_p(stream))
        assert rc == 0, lib.mlq_last_error_message()
        assert lib.mlq_matmul_q8act(w.data_ptr(), qt, xq.data_ptr(), want.data_ptr(), n, k, b) == 0
        torch.cuda.synchronize()
        g, e = got.cpu().numpy(), want.cpu().numpy()
        assert np.all(np.isfinite(g))
        assert O.rel_l2(g, e) < TOL, (call, O.rel_l2(g, e))


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
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())
    # host pointers are refused: this entry point copies nothing
    host_out = np.zeros(n, np.float32)
    rc = lib.mlq_matmul_q8act_noalloc(w.data_ptr(), F.Q8_0, xq.data_ptr(), host_out.ctypes.data, n, k, 1, None)
    assert rc == 1
