"""GPU parity of the quantized GEMV / batch GEMV / dequant / Q8_0 quantizer, called
through the reference-named C-ABI (combined_engine.so) with host numpy buffers and
through mlq_matmul with device buffers, against the pinned oracle.

Tolerance: relative L2 <= 1e-3 for fp32-accumulated products;
bit-exact for dequantization and byte-exact for the Q8_0 quantizer."""
import ctypes
import os

import numpy as np
import pytest

from oracle import formats as F
from oracle import ops as O
from mojollama_b200 import core

pytestmark = pytest.mark.gpu

TOL = 1e-3
QUANT = [F.Q4_0, F.Q4_1, F.Q5_0, F.Q8_0, F.Q4_K, F.Q5_K, F.Q6_K, F.MXFP4, F.MXFP4_REF]
ALL = QUANT + [F.F32, F.F16, F.BF16]
G = os.path.join(os.path.dirname(__file__), "golden")


def cf(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def cu(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8))


@pytest.fixture(scope="module")
def K(cuda_device):
    from mojollama_b200.kernels import load_kernels
    return load_kernels()


def make_w(qt, n, k, seed):
    rng = np.random.default_rng(seed)
    return F.quantize(qt, (rng.standard_normal(n * k) * 0.02).astype(np.float32))


def kdims(qt):
    be = F.BLOCK[qt][0]
    return [k for k in (256, 512, 2048, 2880, 5632) if k % be == 0]


@pytest.mark.parametrize("qt", ALL, ids=lambda q: F.NAMES[q])
def test_quant_matmul_omp_matches_oracle(K, qt):
    for i, (n, k) in enumerate([(1, kdims(qt)[0]), (257, 512), (96, kdims(qt)[-1]), (1031, 2048)]):
        if k % F.BLOCK[qt][0]:
            continue
        w = make_w(qt, n, k, 100 + i)
        x = np.random.default_rng(i).standard_normal(k).astype(np.float32)
        out = np.full(n, np.nan, np.float32)
        # type 39 through the ABI is GGUF MXFP4; the reference's own 17-byte layout is
        # what type 39 means in reference-compat mode
        code = 39 if qt == F.MXFP4_REF else qt
        core().mlq_set_ref_compat(1 if qt == F.MXFP4_REF else 0)
        try:
            K.kern.quant_matmul_omp(cu(w), cf(x), cf(out), n, k, code)
        finally:
            core().mlq_set_ref_compat(0)
        ref = O.gemv(w, qt, x, n, k)[0]
        assert np.all(np.isfinite(out)), (n, k)
        assert O.rel_l2(out, ref) < TOL, (F.NAMES[qt], n, k, O.rel_l2(out, ref))


@pytest.mark.parametrize("qt", QUANT, ids=lambda q: F.NAMES[q])
@pytest.mark.parametrize("B", [2, 3, 4, 5, 8, 13])
def test_batch_matmul_matches_oracle(cuda_device, qt, B):
    lib = cuda_device
    n, k = 300, kdims(qt)[1] if len(kdims(qt)) > 1 else kdims(qt)[0]
    w = make_w(qt, n, k, 7 + B)
    x = np.random.default_rng(B).standard_normal(B * k).astype(np.float32)
    out = np.zeros(B * n, np.float32)
    rc = lib.mlq_matmul(w.ctypes.data, qt, x.ctypes.data, out.ctypes.data, n, k, B)
    assert rc == 0, lib.mlq_last_error_message()
    ref = O.gemv(w, qt, x, n, k)
    assert O.rel_l2(out.reshape(B, n), ref) < TOL


@pytest.mark.parametrize("name,qt", [("q4_0", F.Q4_0), ("q8_0", F.Q8_0), ("q4_k", F.Q4_K), ("q5_k", F.Q5_K),
                                     ("q6_k", F.Q6_K), ("mxfp4", F.MXFP4)])
def test_reference_named_batch_matmul(K, name, qt):
    n, k, B = 130, 512, 3
    w = make_w(qt, n, k, 3)
    x = np.random.default_rng(5).standard_normal(B * k).astype(np.float32)
    out = np.zeros(B * n, np.float32)
    getattr(K.kern, f"{name}_batch_matmul")(cu(w), cf(x), cf(out), n, k, B)
    assert O.rel_l2(out.reshape(B, n), O.gemv(w, qt, x, n, k)) < TOL


def test_matches_reference_c_outputs_from_golden(K):
    # materialise every array once: each NpzFile[key] access returns a fresh temporary
    ro = dict(np.load(os.path.join(G, "ref_ops.npz")))
    n, k, b = (int(v) for v in ro["shape"])
    for qt in (F.Q8_0, F.Q4_0, F.Q4_1, F.Q5_K, F.MXFP4_REF):
        out = np.zeros(n, np.float32)
        rc = core().mlq_matmul(ro[f"gemv_w_{qt}"].ctypes.data, qt, ro[f"gemv_x_{qt}"].ctypes.data,
                               out.ctypes.data, n, k, 1)
        assert rc == 0
        assert O.rel_l2(out, ro[f"gemv_ref_dispatch_{qt}"]) < TOL, F.NAMES[qt]
    for qt in (F.Q8_0, F.Q4_0, F.Q4_K, F.MXFP4_REF):
        out = np.zeros(b * n, np.float32)
        x = np.ascontiguousarray(ro[f"bgemv_x_{qt}"])
        rc = core().mlq_matmul(ro[f"gemv_w_{qt}"].ctypes.data, qt, x.ctypes.data, out.ctypes.data, n, k, b)
        assert rc == 0
        assert O.rel_l2(out.reshape(b, n), ro[f"bgemv_ref_{qt}"]) < TOL, F.NAMES[qt]


@pytest.mark.parametrize("qt", QUANT + [F.BF16, F.F16], ids=lambda q: F.NAMES[q])
def test_dequantize_bit_exact(cuda_device, qt):
    lib = cuda_device
    rng = np.random.default_rng(qt)
    n = 256 * 33
    raw = F.random_blocks(qt, n, rng)
    out = np.zeros(n, np.float32)
    assert lib.mlq_dequantize(raw.ctypes.data, qt, out.ctypes.data, n) == 0
    exp = F.dequantize(qt, raw, n)
    assert np.array_equal(out.view(np.uint32), exp.view(np.uint32))


def test_reference_named_dequantize_rows_match_golden(K):
    fm = np.load(os.path.join(G, "formats.npz"))
    for qt, name in ((F.Q4_K, "q4_k"), (F.Q5_K, "q5_k"), (F.Q6_K, "q6_k"), (F.Q8_0, "q8_0")):
        raw = np.ascontiguousarray(fm[f"deq_raw_{qt}"])
        out = np.zeros(512, np.float32)
        getattr(K.kern, f"{name}_dequantize_row")(cu(raw), cf(out), 512)
        assert np.array_equal(out.view(np.uint32), fm[f"deq_out_{qt}"].view(np.uint32)), name


def test_quantize_row_q8_0_byte_exact(K):
    rng = np.random.default_rng(11)
    x = rng.standard_normal(4096).astype(np.float32)
    x[:32] = 0.0                               # all-zero block: d = 1
    x[32:64] = np.linspace(-1, 1, 32, dtype=np.float32)
    x[64:96] = 1e-30                           # tiny scale
    q = np.zeros(4096 // 32 * 34, np.uint8)
    nb = K.kern.quantize_row_q8_0(cf(x), cu(q), 4096)
    assert nb == 128
    assert np.array_equal(q, F.quantize_q8_0(x))
    fm = np.load(os.path.join(G, "formats.npz"))
    xg = np.ascontiguousarray(fm["quant_x"])
    qg = np.zeros(8 * 34, np.uint8)
    K.kern.quantize_row_q8_0(cf(xg), cu(qg), 256)
    assert np.array_equal(qg, fm["ref_q8_0_bytes"])


def test_q8_0_q8_0_matmul(K):
    n, k, B = 200, 1024, 3
    w = make_w(F.Q8_0, n, k, 1)
    x = np.random.default_rng(2).standard_normal(B * k).astype(np.float32)
    xq = F.quantize_q8_0(x)
    out = np.zeros(B * n, np.float32)
    K.kern.q8_0_q8_0_matmul_omp(cu(w), cu(xq), cf(out), n, k, B)
    xd = F.dequantize(F.Q8_0, xq, B * k)
    assert O.rel_l2(out.reshape(B, n), O.gemv(w, F.Q8_0, xd, n, k)) < TOL


def test_device_pointers_and_unaligned_weights(cuda_device):
    import torch
    lib = cuda_device
    for qt in (F.Q8_0, F.Q4_0, F.MXFP4, F.Q6_K):
        n, k = 515, 512 if F.BLOCK[qt][0] == 256 else 2880
        w = make_w(qt, n, k, 9)
        x = np.random.default_rng(9).standard_normal(2 * k).astype(np.float32)
        for off in (0, 1, 2, 6):          # weights starting at an odd / 2-byte offset
            wd = torch.zeros(w.size + 64, dtype=torch.uint8, device="cuda")
            wd[off:off + w.size] = torch.from_numpy(w).cuda()
            xd = torch.from_numpy(x).cuda()
            od = torch.zeros(2 * n, device="cuda")
            rc = lib.mlq_matmul(wd.data_ptr() + off, qt, xd.data_ptr(), od.data_ptr(), n, k, 2)
            assert rc == 0
            lib.mlq_sync()
            assert O.rel_l2(od.cpu().numpy().reshape(2, n), O.gemv(w, qt, x, n, k)) < TOL, (qt, off)


def test_edge_inputs(cuda_device):
    lib = cuda_device
    n, k = 64, 256
    w = make_w(F.Q4_K, n, k, 4)
    out = np.ones(n, np.float32)
    x = np.zeros(k, np.float32)
    assert lib.mlq_matmul(w.ctypes.data, F.Q4_K, x.ctypes.data, out.ctypes.data, n, k, 1) == 0
    assert np.all(out == 0)
    x[5] = np.nan
    assert lib.mlq_matmul(w.ctypes.data, F.Q4_K, x.ctypes.data, out.ctypes.data, n, k, 1) == 0
    assert np.all(np.isnan(out))        # NaN in -> NaN out, as the reference
    x = np.random.default_rng(0).standard_normal(k).astype(np.float32) * 1e30   # huge range
    assert lib.mlq_matmul(w.ctypes.data, F.Q4_K, x.ctypes.data, out.ctypes.data, n, k, 1) == 0
    assert O.rel_l2(out, O.gemv(w, F.Q4_K, x, n, k)[0]) < TOL
    # K not a multiple of the block: error, output untouched
    out[:] = 7
    assert lib.mlq_matmul(w.ctypes.data, F.Q4_K, x.ctypes.data, out.ctypes.data, n, 100, 1) == 1
    assert np.all(out == 7)


@pytest.mark.parametrize("qt", [F.Q8_0, F.Q4_K, F.Q6_K, F.MXFP4, F.Q4_0, F.Q5_K])
def test_full_size_head_rows_sampled(cuda_device, qt):
    """151936 x 2048 (the output head of BASELINE config 2): every row is checked on
    a sample of rows against the oracle, plus linearity of the whole output."""
    import torch
    lib = cuda_device
    n, k = 151936, 2048
    rng = np.random.default_rng(qt)
    w = F.random_blocks(qt, n * k, rng)
    wd = torch.from_numpy(w).cuda()
    x = rng.standard_normal((2, k)).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    od = torch.zeros(2, n, device="cuda")
    assert lib.mlq_matmul(wd.data_ptr(), qt, xd.data_ptr(), od.data_ptr(), n, k, 2) == 0
    lib.mlq_sync()
    out = od.cpu().numpy()
    rows = np.sort(rng.choice(n, 2048, replace=False))
    rb = F.row_bytes(qt, k)
    wsub = np.concatenate([w[r * rb:(r + 1) * rb] for r in rows])
    assert O.rel_l2(out[:, rows], O.gemv(wsub, qt, x, len(rows), k)) < TOL
    # linearity: W(x0 + x1) == W x0 + W x1
    xs = torch.from_numpy((x[0] + x[1])[None]).cuda()
    os_ = torch.zeros(1, n, device="cuda")
    assert lib.mlq_matmul(wd.data_ptr(), qt, xs.data_ptr(), os_.data_ptr(), n, k, 1) == 0
    lib.mlq_sync()
    assert O.rel_l2(os_.cpu().numpy()[0], out[0] + out[1]) < TOL


def test_host_weight_cache_follows_buffer_contents(cuda_device):
    """A host weight buffer rewritten in place (or freed and re-allocated at the same
    address with the same size) must not be served from a stale device copy."""
    lib = cuda_device
    n, k = 64, 256
    w = make_w(F.Q4_0, n, k, 1)
    x = np.random.default_rng(3).standard_normal(k).astype(np.float32)
    out = np.zeros(n, np.float32)
    assert lib.mlq_matmul(w.ctypes.data, F.Q4_0, x.ctypes.data, out.ctypes.data, n, k, 1) == 0
    assert O.rel_l2(out, O.gemv(w, F.Q4_0, x, n, k)[0]) < TOL
    w[:] = make_w(F.Q4_0, n, k, 2)                   # same address, same size, new contents
    assert lib.mlq_matmul(w.ctypes.data, F.Q4_0, x.ctypes.data, out.ctypes.data, n, k, 1) == 0
    assert O.rel_l2(out, O.gemv(w, F.Q4_0, x, n, k)[0]) < TOL


@pytest.mark.parametrize("qt", [F.Q4_0, F.Q4_K, F.Q5_K, F.Q6_K, F.Q8_0, F.MXFP4, F.Q4_1])
@pytest.mark.parametrize("n", [151899, 20000, 300])
def test_pinned_host_output_written_in_place(cuda_device, qt, n):
    """A pinned host `out` of a one-row product is written by the kernel itself (the
    many-row kernel in one contiguous run per tile).  Every element must be written,
    ragged last tiles included, and equal the device-buffer result bit for bit."""
    import torch
    lib = cuda_device
    k = 2048
    rng = np.random.default_rng(qt * 7 + n)
    wd = torch.from_numpy(F.random_blocks(qt, n * k, rng)).cuda()
    xd = torch.from_numpy(rng.standard_normal(k).astype(np.float32)).cuda()
    od = torch.zeros(n, device="cuda")
    assert lib.mlq_matmul(wd.data_ptr(), qt, xd.data_ptr(), od.data_ptr(), n, k, 1) == 0
    lib.mlq_sync()
    for _ in range(2):   # twice: the second call must not depend on what the first left
        hp = torch.full((n,), float("nan")).pin_memory()
        assert lib.mlq_matmul(wd.data_ptr(), qt, xd.data_ptr(), hp.data_ptr(), n, k, 1) == 0
        assert torch.equal(hp, od.cpu())


@pytest.mark.parametrize("qt", [F.F32, F.F16, F.BF16], ids=lambda q: F.NAMES[q])
@pytest.mark.parametrize("n,k,B", [(128, 2048, 16), (128, 2048, 37), (7, 100, 3), (1000, 512, 1), (3000, 256, 5)])
def test_float_weights_batch(cuda_device, qt, n, k, B):
    """fp32/fp16/bf16 weights (routers, small heads): few rows take one CTA per row for
    up to 16 activation rows per launch (B = 37: three launches), many rows a warp per row;
    K = 100 exercises the scalar path."""
    lib = cuda_device
    w = make_w(qt, n, k, 31 + B)
    x = np.random.default_rng(B + n).standard_normal(B * k).astype(np.float32)
    out = np.full(B * n, np.nan, np.float32)
    rc = lib.mlq_matmul(w.ctypes.data, qt, x.ctypes.data, out.ctypes.data, n, k, B)
    assert rc == 0, lib.mlq_last_error_message()
    assert O.rel_l2(out.reshape(B, n), O.gemv(w, qt, x, n, k)) < TOL


@pytest.mark.parametrize("m,shift", [(1, 0), (1, 1), (3, 0), (40, 0)])
def test_pinned_host_input(cuda_device, m, shift):
    """Activations in pinned host memory: up to 256 KB are read over PCIe by a copy kernel
    (16-byte pieces, or bytes when the buffer is not 16-byte aligned: shift), larger ones by
    the copy engine; the result equals the device-buffer result bit for bit."""
    import torch
    lib = cuda_device
    n, k = 20000, 2048
    rng = np.random.default_rng(m + 10 * shift)
    wd = torch.from_numpy(F.random_blocks(F.Q4_K, n * k, rng)).cuda()
    x = rng.standard_normal(m * k).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    od = torch.zeros(m * n, device="cuda")
    assert lib.mlq_matmul(wd.data_ptr(), F.Q4_K, xd.data_ptr(), od.data_ptr(), n, k, m) == 0
    lib.mlq_sync()
    hx = torch.zeros(m * k + 4).pin_memory()
    hx[shift:shift + m * k] = torch.from_numpy(x)
    for _ in range(2):
        ho = torch.full((m * n,), float("nan")).pin_memory()
        assert lib.mlq_matmul(wd.data_ptr(), F.Q4_K, hx.data_ptr() + 4 * shift, ho.data_ptr(), n, k, m) == 0
        assert torch.equal(ho, od.cpu())


@pytest.mark.parametrize("qt", [F.BF16, F.F16])
@pytest.mark.parametrize("B", [5, 16, 64])
def test_16bit_weights_many_rows(cuda_device, qt, B):
    """bf16 / f16 weights with more than four activation rows (the GPT-OSS attention and head
    shapes at batch 16 / 64): one GEMM over the matrix, activations as two 16-bit parts."""
    import torch
    rng = np.random.default_rng(qt * 100 + B)
    n, k = 4096, 2880
    w = F.quantize(qt, (rng.standard_normal(n * k) * 0.02).astype(np.float32))
    x = rng.standard_normal((B, k)).astype(np.float32)
    dw, dx = torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda()
    out = torch.full((B, n), float("nan"), device="cuda")
    lib = cuda_device
    assert lib.mlq_matmul(dw.data_ptr(), qt, dx.data_ptr(), out.data_ptr(), n, k, B) == 0, \
        lib.mlq_last_error_message()
    torch.cuda.synchronize()
    want = O.gemv(w, qt, x, n, k)
    assert O.rel_l2(out.cpu().numpy(), want) < TOL, O.rel_l2(out.cpu().numpy(), want)
