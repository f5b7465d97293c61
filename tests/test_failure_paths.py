"""Failure paths that need no GPU fault.

CPU: argument checks that run before anything is launched (a corrupt page table of the
paged decode attention, the limits of the bounded-wait self-test).  They return an error
code on a box without a GPU as on one with a GPU, because nothing reaches the device.

GPU: a device-side bounded wait that runs out.  One thread waits on a barrier nothing
arrives on; after its limit it reports the timeout in the status word and the call
returns MLQ_ERR_TIMEOUT.  The word is cleared by that report and the context stays
usable (a matmul afterwards is checked against the oracle)."""
import numpy as np
import pytest

from mojollama_b200 import core
from oracle import formats as F
from oracle import ops as O

MLQ_ERR_ARG, MLQ_ERR_TIMEOUT, MLQ_ERR_CAPACITY = 1, 5, 6


def _paged_call(lib, table, lens, n_pages=8, page_size=16, nh=4, nkh=2, hd=32):
    b = len(lens)
    row = nkh * hd
    pool = np.zeros(n_pages * page_size * row, np.float32)
    q = np.ones(b * nh * hd, np.float32)
    out = np.full(b * nh * hd, 3.0, np.float32)
    seq = np.asarray(lens, np.int32)
    tab = np.ascontiguousarray(table, np.int32)
    rc = lib.mlq_attn_decode_paged(q.ctypes.data, pool.ctypes.data, pool.ctypes.data, tab.ctypes.data,
                                   tab.shape[1], page_size, n_pages, seq.ctypes.data, b, nh, nkh, hd, 0,
                                   out.ctypes.data)
    return rc, out


@pytest.mark.parametrize("bad", [-1, 8, 1 << 20])
def test_paged_attention_rejects_corrupt_page_ids_before_launch(bad):
    """A page id outside [0, n_pages) among the pages a sequence reads is refused on the
    host (MLQ_ERR_ARG) and the output is left untouched."""
    lib = core()
    table = np.array([[0, 1, -1, -1], [2, bad, -1, -1]], np.int32)
    rc, out = _paged_call(lib, table, [20, 17])
    assert rc == MLQ_ERR_ARG, lib.mlq_last_error_message()
    assert b"outside the pool" in lib.mlq_last_error_message()
    assert np.all(out == 3.0)


def test_paged_attention_checks_only_the_pages_a_sequence_reads():
    """Entries past ceil(seq_len / page_size) are not read and may hold anything; with a
    length beyond the table the call is refused with MLQ_ERR_CAPACITY."""
    lib = core()
    table = np.array([[0, 99, 99, 99]], np.int32)
    rc, _ = _paged_call(lib, table, [64 * 4 + 1])
    assert rc == MLQ_ERR_CAPACITY
    # 16 slots = exactly one page: entry 1 (99) is never read, so the table passes the
    # check; on a box without a GPU the call then fails only at the device stage
    lib.mlq_clear_error()
    rc, _ = _paged_call(lib, table, [16])
    assert rc != MLQ_ERR_ARG or b"outside the pool" not in lib.mlq_last_error_message()


def test_wait_selftest_limits_are_checked():
    lib = core()
    assert lib.mlq_selftest_wait_timeout(0) == MLQ_ERR_ARG
    assert lib.mlq_selftest_wait_timeout(2000000) == MLQ_ERR_ARG


@pytest.mark.gpu
def test_bounded_wait_runs_out_and_reports_timeout(cuda_device):
    import torch
    lib = cuda_device
    assert lib.mlq_device_status() == 0
    rc = lib.mlq_selftest_wait_timeout(20000)            # 20 ms limit
    assert rc == MLQ_ERR_TIMEOUT, lib.mlq_last_error_message()
    assert b"gave up" in lib.mlq_last_error_message()
    assert lib.mlq_device_status() == 0                   # the report cleared the word
    # the context is still usable
    n, k = 256, 2048
    rng = np.random.default_rng(5)
    w = F.quantize(F.Q8_0, (rng.standard_normal(n * k) * 0.02).astype(np.float32))
    x = rng.standard_normal(k).astype(np.float32)
    out = np.zeros(n, np.float32)
    assert lib.mlq_matmul(w.ctypes.data, F.Q8_0, x.ctypes.data, out.ctypes.data, n, k, 1) == 0
    assert O.rel_l2(out, O.gemv(w, F.Q8_0, x, n, k)[0]) < 1e-3
    torch.cuda.synchronize()
