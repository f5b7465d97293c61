"""batch_forward / moe_ffn (cengine_batch_instr.c:1233-1493, 591-665) on the GPU.

Default mode is checked against the numpy model oracle (oracle/model.py: the batch
engine's layer structure with the normalised activations feeding the projections).
Reference-compatibility mode (mlq_set_ref_compat(1)) reproduces the reference's own data
flow and is checked against the reference C engine built from its sources
(oracle/_ref/libref_engine.so) on the same BC bytes, step by step.
Bars: every operation inside the step meets the per-op bar (relative L2 <= 1e-3, checked
op by op in the other GPU test files); the logits and hidden states of a whole step, a
composition of up to three layers of such ops (the tensor-core GEMM rounds weights and
activations to fp16 when a batch takes it), are held to MODEL_TOL = 3e-3; greedy tokens
identical where the oracle's top-2 margin exceeds 1e-2; KV pages, page tables and sequence
lengths as the reference keeps them."""
import ctypes

import numpy as np
import pytest

from mojollama_b200 import bc as BCm
from oracle import model as OM
from oracle import ops as O
from oracle import ref as R

from model_fixture import fill_bc, make_model, ws_stride

pytestmark = pytest.mark.gpu
TOL = 1e-3          # one operation (KV rows, the MoE block, the SSM state)
MODEL_TOL = 3e-3    # logits / hidden state after a whole step (three layers of TOL-bounded ops)


def dev_to_np(ptr, n):
    import torch

    class _A:
        pass

    a = _A()
    a.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (int(ptr), False), "version": 2}
    torch.cuda.synchronize()
    return torch.as_tensor(a, device="cuda").cpu().numpy().copy()


def greedy_ok(got, ref):
    for g, r in zip(np.atleast_2d(got), np.atleast_2d(ref)):
        top = np.argsort(r)[::-1]
        if r[top[0]] - r[top[1]] > 1e-2:
            assert int(np.argmax(g)) == int(top[0])


def _run_default(cuda_device, m, schedule, page_size=None, n_pages=None, seed=0):
    """schedule: list of lists of sequence indices taking one token each step."""
    n_seq = 1 + max(max(s) for s in schedule)
    caches = [BCm.KVCache(m["L"], m["NKH"], m["HD"], page_size=page_size, n_pages=n_pages) for _ in range(n_seq)]
    st = OM.new_state(m, n_seq)
    ssm = np.zeros((m["L"], OM.SSM_GROUPS, OM.SSM_STATE), np.float32)
    rng = np.random.default_rng(seed)
    bld = BCm.BCBuilder()
    logits = np.zeros(64 * m["V"], np.float32)
    fill_bc(m, bld, [caches[0].block], logits, ssm_state=ssm)
    for step, seqs in enumerate(schedule):
        B = len(seqs)
        toks = rng.integers(0, m["V"], B).astype(np.int32)
        bld.kv_array([caches[s].block for s in seqs])
        ws = np.zeros(12 * B * ws_stride(m, B), np.float32)
        BCm.batch_forward(bld.bc, toks, ws)
        want, hid = OM.forward_step(m, st, seqs, toks)
        got = logits[:B * m["V"]].reshape(B, m["V"])
        assert O.rel_l2(got, want) < MODEL_TOL, (step, O.rel_l2(got, want))
        assert O.rel_l2(ws[:B * m["N"]].reshape(B, -1), hid) < MODEL_TOL
        greedy_ok(got, want)
        first_attn = [i for i, ly in enumerate(m["layers"]) if ly["type"] == "attn"][0]
        for s in seqs:
            assert caches[s].seq_len == len(st["kv"][s][first_attn][0])
        if any(ly["type"] == "ssm" for ly in m["layers"]):
            assert O.rel_l2(ssm, st["ssm"]) < TOL
    return caches, st


def test_dense_forward_matches_oracle(cuda_device):
    m = make_model("dense", seed=1)
    sched = [[0, 1], [0, 1], [0, 1, 2], [0, 1, 2], [2, 0], [1, 2, 0], [0, 1, 2]]
    # 4-slot pages so the steps cross page boundaries
    _run_default(cuda_device, m, sched, page_size=4, n_pages=16)


def test_hybrid_moe_forward_matches_oracle(cuda_device):
    m = make_model("hybrid", seed=2)
    _run_default(cuda_device, m, [[0, 1, 2]] * 4 + [[1]], seed=3)


def test_forward_kv_pages_and_mirror(cuda_device):
    """K/V rows land in the page pool ([L][n_pages][64][row] K, then V) and in the
    KVBlock's own k/v arrays, at the page the LIFO free list hands out (0 first)."""
    m = make_model("dense", seed=4, attn_modes=["sep", "qk", "sep"])
    caches, st = _run_default(cuda_device, m, [[0, 1]] * 3, seed=5)
    L, kvrow = m["L"], m["NKH"] * m["HD"]
    for s, c in enumerate(caches):
        blk = c.block
        assert blk.pt.table[0] == 0 and blk.pt.free_count == blk.pt.n_pages - 1
        n_pool = L * blk.pt.n_pages * 64 * kvrow
        pages = dev_to_np(ctypes.cast(blk.pt.pages, ctypes.c_void_p).value, 2 * n_pool)
        mk = dev_to_np(ctypes.cast(blk.k, ctypes.c_void_p).value, L * 1024 * 64 * kvrow)
        for l in range(L):
            ks, vs = st["kv"][s][l]
            for p in range(len(ks)):
                off = (l * blk.pt.n_pages * 64 + p) * kvrow
                assert O.rel_l2(pages[off:off + kvrow], ks[p]) < TOL
                assert O.rel_l2(pages[n_pool + off:n_pool + off + kvrow], vs[p]) < TOL
                moff = (l * 1024 * 64 + p) * kvrow
                assert O.rel_l2(mk[moff:moff + kvrow], ks[p]) < TOL


def test_forward_rejects_bad_inputs(cuda_device):
    m = make_model("dense", seed=6, attn_modes=["sep", "sep", "sep"])
    lib = cuda_device
    c = BCm.KVCache(m["L"], m["NKH"], m["HD"])
    bld = BCm.BCBuilder()
    logits = np.full(m["V"], 7.0, np.float32)
    fill_bc(m, bld, [c.block], logits)
    tok = np.zeros(65, np.int32)
    assert lib.mlq_batch_forward(ctypes.byref(bld.bc), tok.ctypes.data, 0, None) != 0
    assert lib.mlq_batch_forward(ctypes.byref(bld.bc), tok.ctypes.data, 65, None) != 0
    # a KVBlock whose page pool is host memory (not made by this library) is refused
    host = BCm.KVBlock()
    pages = np.zeros(16, np.float32)
    table = np.full(1024, -1, np.int32)
    host.pt.page_size, host.pt.n_pages, host.pt._nkh, host.pt._hd, host.pt._n_layers = 64, 1, m["NKH"], m["HD"], m["L"]
    host.pt.pages = pages.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    host.pt.table = table.ctypes.data_as(ctypes.POINTER(ctypes.c_int))
    bld.kv_array([host])
    assert lib.mlq_batch_forward(ctypes.byref(bld.bc), tok.ctypes.data, 1, None) != 0
    assert np.all(logits == 7.0) and host.seq_len[0] == 0
    # a sequence at max_ctx is refused
    bld.kv_array([c.block])
    c.block.seq_len[0] = m["max_ctx"]
    assert lib.mlq_batch_forward(ctypes.byref(bld.bc), tok.ctypes.data, 1, None) != 0
    c.block.seq_len[0] = 0


def test_moe_ffn_matches_oracle(cuda_device):
    """moe_ffn (cengine_batch_instr.c:591): router, softmax, top-k (no renormalisation),
    SiLU(gate)*up without a clamp, weighted sum; one row per token here."""
    m = make_model("hybrid", seed=7)
    bld = BCm.BCBuilder()
    c = BCm.KVCache(m["L"], m["NKH"], m["HD"])
    fill_bc(m, bld, [c.block], np.zeros(m["V"], np.float32))
    lib = BCm.core()
    from mojollama_b200.kernels import load_kernels
    k = load_kernels()
    rng = np.random.default_rng(8)
    B, N = 5, m["N"]
    x = (rng.standard_normal((B, N)) * 2).astype(np.float32)
    ffn = np.zeros((B, N), np.float32)
    mo = m["moe"]
    lib.mlq_clear_error()
    for l in range(m["L"]):
        k.cengine.moe_ffn(ctypes.byref(bld.bc), l, x.ctypes.data, None, None, ffn.ctypes.data, B)
        assert lib.mlq_last_error() == 0
        ly = m["layers"][l]
        for b in range(B):
            idx, w = O.router_topk(ly["router"].astype(np.float64) @ x[b].astype(np.float64), mo["k"], False)
            want = O.moe_forward(ly["gate_exps"], ly["up_exps"], ly["down_exps"], (mo["gq"], mo["uq"], mo["dq"]),
                                 x[b], mo["M"], N, idx, w, clamp=False)
            assert O.rel_l2(ffn[b], want) < TOL


# ------------------------------------------------------------------ reference compatibility
needs_ref = pytest.mark.skipif(not R.available(), reason="reference build (oracle/_ref) not present")


def _run_compat(cuda_device, m, B, steps, seed):
    lib = cuda_device
    ref = R.RefEngine()
    S = ws_stride(m, B)
    rng = np.random.default_rng(seed)
    xn_region = (rng.standard_normal(B * m["N"]) * 0.7).astype(np.float32)
    L, V, N = m["L"], m["V"], m["N"]
    kvrow = m["NKH"] * m["HD"]
    # reference side: its own kv_init (host memory), its own buffers
    ref_kv = [BCm.KVBlock() for _ in range(B)]
    for kv in ref_kv:
        ref.so.kv_init(ctypes.byref(kv), L, m["NKH"], m["HD"])
    ref_logits = np.zeros(B * V, np.float32)
    ref_ssm = np.zeros(L * OM.SSM_GROUPS * OM.SSM_STATE, np.float32)
    ref_work = np.zeros(m["max_ctx"] * kvrow * 2 + 4096, np.float32)
    rb = BCm.BCBuilder()
    fill_bc(m, rb, ref_kv, ref_logits, ssm_state=ref_ssm, workspace=ref_work)
    ours = [BCm.KVCache(L, m["NKH"], m["HD"]) for _ in range(B)]
    logits = np.zeros(B * V, np.float32)
    ssm = np.zeros_like(ref_ssm)
    ob = BCm.BCBuilder()
    fill_bc(m, ob, [c.block for c in ours], logits, ssm_state=ssm)
    assert lib.mlq_set_ref_compat(1) == 0
    try:
        for step in range(steps):
            toks = rng.integers(0, V, B).astype(np.int32)
            ws_ref = np.zeros(12 * B * S, np.float32)
            ws_ref[B * S:B * S + B * N] = xn_region
            ws = ws_ref.copy()
            ref.so.batch_forward(ctypes.byref(rb.bc), toks.ctypes.data, B, ws_ref.ctypes.data)
            BCm.batch_forward(ob.bc, toks, ws)
            assert O.rel_l2(logits, ref_logits) < TOL, (step, O.rel_l2(logits, ref_logits))
            assert O.rel_l2(ws[:B * N], ws_ref[:B * N]) < TOL
            assert np.array_equal(ws[B * S:B * S + B * N], xn_region)
            greedy_ok(logits.reshape(B, V), ref_logits.reshape(B, V))
            assert O.rel_l2(ssm, ref_ssm) < TOL
            for c, kv in zip(ours, ref_kv):
                assert c.block.seq_len[0] == kv.seq_len[0] == step + 1
                assert c.block.pt.free_count == kv.pt.free_count
                assert [c.block.pt.table[i] for i in range(4)] == [kv.pt.table[i] for i in range(4)]
        # the page pools hold the same K/V rows
        for c, kv in zip(ours, ref_kv):
            n_pool = L * kv.pt.n_pages * 64 * kvrow
            got = dev_to_np(ctypes.cast(c.block.pt.pages, ctypes.c_void_p).value, 2 * n_pool)
            want = np.ctypeslib.as_array(kv.pt.pages, shape=(2 * n_pool,))
            for l in range(L):
                for half in (0, n_pool):
                    off = half + l * kv.pt.n_pages * 64 * kvrow
                    if np.any(want[off:off + steps * kvrow]):
                        assert O.rel_l2(got[off:off + steps * kvrow], want[off:off + steps * kvrow]) < TOL
    finally:
        lib.mlq_set_ref_compat(0)


@needs_ref
def test_ref_compat_dense_matches_reference_build(cuda_device):
    _run_compat(cuda_device, make_model("dense", seed=9, attn_modes=["sep", "qk", "sep"]), B=2, steps=4, seed=10)


@needs_ref
def test_ref_compat_hybrid_moe_matches_reference_build(cuda_device):
    _run_compat(cuda_device, make_model("hybrid", seed=11), B=2, steps=3, seed=12)


@needs_ref
def test_ref_compat_fused_qkv_matches_reference_build(cuda_device):
    """The reference's fused-QKV split (8192 rows; sequence b's Q read at b*NH*HD)."""
    _run_compat(cuda_device, make_model("qkv8192", seed=13), B=2, steps=2, seed=14)
