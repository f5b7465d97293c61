"""GPU parity of decode attention: flat KV through the reference-named entry points
(gqa_attention.so gqa_attention_decode, combined_engine.so gqa, simd_ops.so
attention_forward), split-K and sliding-window variants, and paged KV through the
reference's PageTable (page_table_init / alloc / map_page) -- against the oracle's
exact softmax attention.  Tolerance: relative L2 <= 1e-3 (fp32 accumulate)."""
import ctypes

import numpy as np
import pytest

from oracle import ops as O

pytestmark = pytest.mark.gpu
TOL = 1e-3
cf = ctypes.POINTER(ctypes.c_float)
ci = ctypes.c_int


def p(a):
    return a.ctypes.data_as(cf)


@pytest.fixture(scope="module")
def libs(cuda_device):
    from mojollama_b200 import load_alias
    g = load_alias("gqa_attention.so")
    g.gqa_attention_decode.argtypes = [cf, cf, cf, cf, ci, ci, ci, ci, cf]
    e = load_alias("combined_engine.so")
    e.gqa.argtypes = [cf, cf, cf, cf, ci, ci, ci, ci]
    s = load_alias("simd_ops.so")
    s.attention_forward.argtypes = [cf, cf, cf, cf, ci, ci, ci, ci, ci]
    s.kv_cache_update.argtypes = [cf, cf, cf, cf, ci, ci, ci, ci, ci]
    return g, e, s, cuda_device


SHAPES = [(32, 4, 64, 1), (32, 4, 64, 77), (32, 4, 128, 1000), (64, 8, 64, 4096), (16, 2, 256, 300),
          (8, 8, 80, 33), (32, 4, 96, 65)]


def rand_case(nh, nkh, hd, sl, seed):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal(nh * hd).astype(np.float32)
    k = rng.standard_normal(sl * nkh * hd).astype(np.float32)
    v = rng.standard_normal(sl * nkh * hd).astype(np.float32)
    return q, k, v


@pytest.mark.parametrize("nh,nkh,hd,sl", SHAPES)
def test_gqa_attention_decode_flat(libs, nh, nkh, hd, sl):
    g, e, s, _ = libs
    q, k, v = rand_case(nh, nkh, hd, sl, sl)
    ref = O.gqa_decode(q, k, v, nh, nkh, hd)
    out = np.full(nh * hd, np.nan, np.float32)
    ws = np.zeros(1, np.float32)
    g.gqa_attention_decode(p(q), p(k), p(v), p(out), sl, nh, nkh, hd, p(ws))
    assert O.rel_l2(out, ref) < TOL
    out2 = np.full(nh * hd, np.nan, np.float32)
    e.gqa(p(out2), p(q), p(k), p(v), sl, nh, nkh, hd)
    assert O.rel_l2(out2, ref) < TOL


def test_attention_forward_and_kv_cache_update(libs):
    _, _, s, _ = libs
    nh, nkh, hd, max_seq = 32, 4, 64, 64
    rng = np.random.default_rng(3)
    kc = np.zeros(max_seq * nkh * hd, np.float32)
    vc = np.zeros_like(kc)
    for pos in range(10):
        kn = rng.standard_normal(nkh * hd).astype(np.float32)
        vn = rng.standard_normal(nkh * hd).astype(np.float32)
        s.kv_cache_update(p(kc), p(vc), p(kn), p(vn), 0, pos, max_seq, nkh, hd)
    q = rng.standard_normal(nh * hd).astype(np.float32)
    out = np.zeros(nh * hd, np.float32)
    s.attention_forward(p(q), p(kc), p(vc), p(out), nh, nkh, hd, 9, max_seq)
    ref = O.gqa_decode(q, kc[:10 * nkh * hd], vc[:10 * nkh * hd], nh, nkh, hd)
    assert O.rel_l2(out, ref) < TOL


@pytest.mark.parametrize("window", [1, 128, 5000])
def test_sliding_window(libs, window):
    _, _, _, lib = libs
    nh, nkh, hd, sl = 64, 8, 64, 1500
    q, k, v = rand_case(nh, nkh, hd, sl, window)
    out = np.zeros(nh * hd, np.float32)
    assert lib.mlq_attn_decode_flat(q.ctypes.data, k.ctypes.data, v.ctypes.data, out.ctypes.data, sl, nh, nkh, hd,
                                    window) == 0
    assert O.rel_l2(out, O.gqa_decode(q, k, v, nh, nkh, hd, window)) < TOL


@pytest.mark.parametrize("page_size", [16, 64])
def test_paged_decode_through_reference_page_table(libs, page_size):
    """Three sequences of different lengths share one page pool; pages are handed out
    by the reference's LIFO allocator interleaved across sequences, so logical pages map
    to scattered physical pages."""
    import torch
    _, eng, _, lib = libs
    from tests.test_layouts import PageTable
    eng.page_table_init.argtypes = [ctypes.POINTER(PageTable), ci, ci, ci, ci, ci]
    eng.page_table_alloc.argtypes = [ctypes.POINTER(PageTable)]
    eng.page_table_alloc.restype = ci
    nh, nkh, hd, n_layers, n_pages = 32, 4, 128, 1, 64
    row = nkh * hd
    pt = PageTable()
    eng.page_table_init(ctypes.byref(pt), n_pages, page_size, nkh, hd, n_layers)
    assert pt.n_pages == n_pages and pt.free_count == n_pages
    lens = [page_size * 3 + 5, 1, page_size * 2]
    tables = np.full((3, 16), -1, np.int32)
    rng = np.random.default_rng(page_size)
    oracle = O.PagedKV(n_pages, page_size, row)
    pool_k = torch.zeros(n_pages * page_size * row, device="cuda")
    pool_v = torch.zeros_like(pool_k)
    # allocate round-robin so the sequences' pages interleave in the pool
    for blk in range(max((l + page_size - 1) // page_size for l in lens)):
        for b, l in enumerate(lens):
            if blk * page_size < l:
                phys = eng.page_table_alloc(ctypes.byref(pt))
                assert phys == oracle.alloc()
                tables[b, blk] = phys
                oracle.tables.setdefault(b, {})[blk] = phys
    for b, l in enumerate(lens):
        for pos in range(l):
            kr = rng.standard_normal(row).astype(np.float32)
            vr = rng.standard_normal(row).astype(np.float32)
            phys, off = tables[b, pos // page_size], pos % page_size
            base = (phys * page_size + off) * row
            pool_k[base:base + row] = torch.from_numpy(kr).cuda()
            pool_v[base:base + row] = torch.from_numpy(vr).cuda()
            oracle.k[phys, off] = kr
            oracle.v[phys, off] = vr
    q = rng.standard_normal((3, nh * hd)).astype(np.float32)
    out = np.zeros((3, nh * hd), np.float32)
    seq = np.array(lens, np.int32)
    torch.cuda.synchronize()
    rc = lib.mlq_attn_decode_paged(q.ctypes.data, pool_k.data_ptr(), pool_v.data_ptr(), tables.ctypes.data, 16,
                                   page_size, n_pages, seq.ctypes.data, 3, nh, nkh, hd, 0, out.ctypes.data)
    assert rc == 0, lib.mlq_last_error_message()
    for b, l in enumerate(lens):
        ks, vs = oracle.gather(b, l)
        assert O.rel_l2(out[b], O.gqa_decode(q[b], ks, vs, nh, nkh, hd)) < TOL, b
    lib.mlq_page_table_destroy(ctypes.addressof(pt))
